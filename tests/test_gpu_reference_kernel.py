"""kernel-lab's own CUDA kernels on the same GPU: a second checker and the comparator.

``oracle/build_ref.py`` compiles kernel-lab's csrc/paged_attention.cu and csrc/rmsnorm.cu,
unmodified, for sm_100a into ``oracle/_ref/`` (test infrastructure, git-ignored, built where
the reference tree is present and shipped with the repository's other built files). These
tests

1. run kernel-lab's own GPU kernels on the golden cases they support and check them against
   the golden outputs (made by kernel-lab's CPU reference) and against this repository's
   kernels, so the parity chain covers the reference's GPU code as well as its CPU code;
2. time kernel-lab's kernels and this repository's on the benchmark configurations, with
   PyTorch's gather + scaled-dot-product attention (the comparator kernel-lab's own bench
   uses, kernel_lab/bench/__main__.py:128-139) and FlashInfer's batch paged decode (kernel-lab's
   bench row, __main__.py:142-169, on the installed 0.6 API) beside them, print one
   ``COMPARATOR {json}`` line per configuration, and assert that the B200 kernels are the
   fastest there.

Skipped when the comparator library was not built.
"""

from __future__ import annotations

import ctypes
import json

import numpy as np

import pytest
import torch
import torch.nn.functional as F

from tests.conftest import (
    DT,
    REPO,
    build_decode_case,
    golden_array,
    golden_index,
    golden_to_torch,
    make_rms_inputs,
    tolerance,
)

from kernel_lab import cuda_ops  # noqa: E402,F401  (registers torch.ops.kernel_lab)

REF_LIB = REPO / "oracle" / "_ref" / "libkernel_lab_ref.so"
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not REF_LIB.exists(), reason="kernel-lab comparator not built (oracle/build_ref.py)"),
]

_lib = None


def ref_lib():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(REF_LIB))
        vp, i, i64, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        lib.klref_paged_decode_attention.restype = i
        lib.klref_paged_decode_attention.argtypes = [i, vp, vp, vp, vp, vp, vp, i, i, i, i, i, i64, f, vp]
        lib.klref_rms_norm.restype = i
        lib.klref_rms_norm.argtypes = [i, vp, vp, vp, vp, i, i, i64, f, vp]
        _lib = lib
    return _lib


CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def ref_decode(out, q, kv, scale=None) -> int:
    """kernel-lab's launch_paged_decode_attention on the current stream; returns its cudaError_t."""
    b, hq, d = q.shape
    _, page, hkv, _ = kv.k_cache.shape
    return ref_lib().klref_paged_decode_attention(
        CODE[q.dtype], out.data_ptr(), q.data_ptr(), kv.k_cache.data_ptr(), kv.v_cache.data_ptr(),
        kv.block_table.data_ptr(), kv.seq_lens.data_ptr(), b, hq, hkv, d, page, kv.block_table.stride(0),
        d**-0.5 if scale is None else scale, torch.cuda.current_stream().cuda_stream,
    )


def ref_fused_add_rms_norm(out, x, res, w, eps) -> int:
    return ref_lib().klref_rms_norm(
        CODE[x.dtype], out.data_ptr(), x.data_ptr(), res.data_ptr(), w.data_ptr(), x.shape[0], x.shape[1],
        x.stride(0), eps, torch.cuda.current_stream().cuda_stream,
    )


def ours_decode(out, q, kv, scale=None):
    torch.ops.kernel_lab.paged_decode_attention(out, q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens,
                                                q.shape[-1] ** -0.5 if scale is None else scale)


def sdpa_decode(q, kv, ctx):
    """Gather every sequence's pages, then PyTorch attention (all sequences have length ctx)."""
    b, hq, d = q.shape
    _, page, hkv, _ = kv.k_cache.shape
    pages = ctx // page
    ids = kv.block_table[:, :pages].long()
    k = kv.k_cache[ids].reshape(b, pages * page, hkv, d).transpose(1, 2)
    v = kv.v_cache[ids].reshape(b, pages * page, hkv, d).transpose(1, 2)
    return F.scaled_dot_product_attention(q.unsqueeze(2), k, v, scale=d**-0.5, enable_gqa=True).squeeze(2)


# FlashInfer 0.6's batch decode configurations: its CUDA-core kernel (the default, as kernel-lab's
# bench plans it), its tensor-core kernel (use_tensor_cores=True, FlashInfer's choice for GQA),
# and its Blackwell backend (backend="trtllm-gen", precompiled TensorRT-LLM kernels).
FLASHINFER_VARIANTS = {
    "flashinfer_fa2": {},
    "flashinfer_tensor_cores": {"use_tensor_cores": True},
    "flashinfer_trtllm_gen": {"backend": "trtllm-gen"},
}


def flashinfer_decode(q, kv, ctx, variant="flashinfer_fa2"):
    """FlashInfer's batch paged decode (library comparator, NHD pages as here) in one of
    FLASHINFER_VARIANTS, or None when that configuration does not run on this box."""
    try:
        import flashinfer

        b, hq, d = q.shape
        _, page, hkv, _ = kv.k_cache.shape
        pages = ctx // page
        indptr = torch.arange(0, b + 1, device=q.device, dtype=torch.int32) * pages
        indices = kv.block_table[:, :pages].reshape(-1).contiguous()
        last = torch.full((b,), page, dtype=torch.int32, device=q.device)
        ws = torch.zeros(256 << 20, dtype=torch.uint8, device=q.device)
        wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD", **FLASHINFER_VARIANTS[variant])
        plan_kw = {}
        if FLASHINFER_VARIANTS[variant].get("backend") == "trtllm-gen":
            plan_kw = dict(block_tables=kv.block_table[:, :pages].contiguous(),
                           seq_lens=torch.full((b,), ctx, dtype=torch.int32, device=q.device))
        wrapper.plan(indptr, indices, last, hq, hkv, d, page, q_data_type=q.dtype, kv_data_type=q.dtype, **plan_kw)
        out = wrapper.run(q, (kv.k_cache, kv.v_cache))
        return lambda: wrapper.run(q, (kv.k_cache, kv.v_cache), out=out), out
    except Exception as exc:  # a comparator that does not run is reported, not failed
        print(f"COMPARATOR {variant} unavailable: {type(exc).__name__}: {str(exc)[:200]}")
        return None


def device_us(fn, iters: int, warmup: int = 3) -> float:
    """Mean device time per call of `iters` back-to-back calls (CUDA events, current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


# Golden cases inside kernel-lab's CUDA support (head_dim 64/128/256, group 1/2/4/8).
SUPPORTED = [
    c["name"] for c in golden_index()["decode"]
    if c["d"] in (64, 128, 256) and c["hq"] // c["hkv"] in (1, 2, 4, 8)
]


@pytest.mark.parametrize("name", SUPPORTED)
def test_reference_kernel_agrees_with_golden_and_with_ours(name):
    case = next(c for c in golden_index()["decode"] if c["name"] == name)
    dt = DT[case["dt"]]
    q, kv, _, _ = build_decode_case(case, device="cuda")
    theirs = torch.full_like(q, float("nan"))
    assert ref_decode(theirs, q, kv, case.get("scale")) == 0
    ours = torch.full_like(q, float("nan"))
    ours_decode(ours, q, kv, case.get("scale"))
    torch.cuda.synchronize()
    want = golden_to_torch(golden_array("decode", f"{name}/out"), case["dt"]).cuda()
    torch.testing.assert_close(theirs, want, **tolerance(dt))
    # Both within kernel-lab's tolerance of each other (each rounds once from fp32 math).
    torch.testing.assert_close(ours, theirs, **tolerance(dt))


def test_reference_kernel_rejects_mqa_that_ours_runs():
    """kernel-lab's launcher returns cudaErrorInvalidValue for group 32 (paged_attention.cu:130-199);
    the B200 op runs it (config 4's MQA layout)."""
    case = next(c for c in golden_index()["decode"] if c["name"] == "cfg4_32_1")
    q, kv, _, _ = build_decode_case(case, device="cuda")
    assert ref_decode(torch.empty_like(q), q, kv) == 1
    ours = torch.empty_like(q)
    ours_decode(ours, q, kv)
    want = golden_to_torch(golden_array("decode", "cfg4_32_1/out"), "bf16").cuda()
    torch.testing.assert_close(ours, want, **tolerance(torch.bfloat16))


def _report(name: str, algorithmic_bytes: int, times: dict[str, float]) -> None:
    line = {"config": name, "algorithmic_bytes": algorithmic_bytes,
            "us": {k: round(v, 1) for k, v in times.items()},
            "GBps": {k: round(algorithmic_bytes / v / 1e3) for k, v in times.items()}}
    print("COMPARATOR " + json.dumps(line))


DECODE_CONFIGS = [
    # (name, batch, ctx, hq, hkv, asserted)
    ("cfg3_llama3_8b_b64_ctx4096", 64, 4096, 32, 8, True),
    ("cfg3_llama3_8b_b8_ctx4096", 8, 4096, 32, 8, False),
    ("cfg3_llama3_8b_b64_ctx512", 64, 512, 32, 8, False),
    ("cfg3_llama3_8b_b1_ctx512", 1, 512, 32, 8, False),
    ("cfg5_llama3_70b_b256_ctx8192", 256, 8192, 64, 8, True),
]


@pytest.mark.parametrize("name,batch,ctx,hq,hkv,asserted", DECODE_CONFIGS)
def test_decode_against_kernel_lab_and_torch_on_the_same_gpu(name, batch, ctx, hq, hkv, asserted):
    from kernel_lab.kv_cache import random_paged_pool
    from kernel_lab.roofline import decode_attention_work

    q, kv = random_paged_pool([ctx] * batch, hq, hkv, 128, 16, dtype=torch.bfloat16, device="cuda", seed=11)
    ours, theirs = torch.empty_like(q), torch.empty_like(q)
    ours_decode(ours, q, kv)
    assert ref_decode(theirs, q, kv) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(ours, theirs, **tolerance(torch.bfloat16))
    work = decode_attention_work([ctx] * batch, hq, hkv, 128, 2).bytes
    iters = max(5, min(100, int(2e10 // work)))
    times = {
        "b200": device_us(lambda: ours_decode(ours, q, kv), iters),
        "kernel_lab_cuda": device_us(lambda: ref_decode(theirs, q, kv), max(3, iters // 4)),
    }
    if batch * ctx <= 64 * 4096:  # the gather copies the whole context once more
        times["torch_gather_sdpa"] = device_us(lambda: sdpa_decode(q, kv, ctx), max(3, iters // 4))
    for variant in FLASHINFER_VARIANTS:
        fi = flashinfer_decode(q, kv, ctx, variant)
        if fi is None:
            continue
        run, fi_out = fi
        torch.cuda.synchronize()
        torch.testing.assert_close(fi_out, ours, **tolerance(torch.bfloat16))
        times[variant] = device_us(run, max(3, iters // 2))
        del fi, run, fi_out
    _report(name, work, times)
    if asserted:  # faster than kernel-lab's own kernel and the PyTorch path; FlashInfer is reported
        assert times["b200"] < min(v for k, v in times.items() if not k.startswith(("b200", "flashinfer")))


@pytest.mark.parametrize("rows,hidden", [(4096, 8192), (4096, 4096), (16, 8192)])
def test_fused_add_rms_norm_against_kernel_lab_on_the_same_gpu(rows, hidden):
    from kernel_lab.roofline import rms_norm_work

    x, r, w = (t.cuda() for t in make_rms_inputs((rows, hidden), torch.bfloat16, seed=3))
    res_ours, res_theirs = r.clone(), r.clone()
    out_ours, out_theirs = torch.empty_like(x), torch.empty_like(x)
    torch.ops.kernel_lab.fused_add_rms_norm(out_ours, x, res_ours, w, 1e-5)
    assert ref_fused_add_rms_norm(out_theirs, x, res_theirs, w, 1e-5) == 0
    torch.cuda.synchronize()
    assert torch.equal(res_ours, res_theirs)  # the residual sum is bit-exact in both
    # kernel-lab takes rsqrtf, this repository IEEE 1/sqrt: within kernel-lab's own tolerance.
    torch.testing.assert_close(out_ours, out_theirs, **tolerance(torch.bfloat16))
    res_a, res_b = r.clone(), r.clone()
    times = {
        "b200": device_us(lambda: torch.ops.kernel_lab.fused_add_rms_norm(out_ours, x, res_a, w, 1e-5), 100),
        "kernel_lab_cuda": device_us(lambda: ref_fused_add_rms_norm(out_theirs, x, res_b, w, 1e-5), 100),
    }
    _report(f"rmsnorm_fused_{rows}x{hidden}_bf16", rms_norm_work(rows, hidden, 2, True).bytes, times)
    if rows >= 4096:
        assert times["b200"] < times["kernel_lab_cuda"]


def flashinfer_cascade(q, kv):
    """FlashInfer's two-level cascade (shared-prefix prefill per group + per-sequence decode,
    merged by LSE), or None when its API does not run on this box."""
    try:
        import flashinfer

        b, hq, d = q.shape
        _, page, hkv, _ = kv.k_cache.shape
        dev = q.device

        def level(rows, lens):
            npages = [-(-int(n) // page) for n in lens]
            indptr = torch.tensor([0, *np.cumsum(npages).tolist()], dtype=torch.int32, device=dev)
            indices = torch.cat([rows[i, :n] for i, n in enumerate(npages)]).contiguous()
            last = torch.tensor([int(n) - (p - 1) * page for n, p in zip(lens, npages)], dtype=torch.int32, device=dev)
            return indptr, indices, last

        p_indptr, p_idx, p_last = level(kv.prefix_block_table, kv.prefix_lens.tolist())
        s_indptr, s_idx, s_last = level(kv.block_table, kv.seq_lens.tolist())
        ws = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        wrapper = flashinfer.MultiLevelCascadeAttentionWrapper(2, ws, "NHD")
        wrapper.plan([kv.prefix_indptr, torch.arange(b + 1, dtype=torch.int32, device=dev)], [p_indptr, s_indptr],
                     [p_idx, s_idx], [p_last, s_last], hq, hkv, d, page, q_data_type=q.dtype, kv_data_type=q.dtype)
        out = wrapper.run(q, (kv.k_cache, kv.v_cache))
        return lambda: wrapper.run(q, (kv.k_cache, kv.v_cache)), out
    except Exception as exc:  # a comparator that does not run is reported, not failed
        print(f"COMPARATOR flashinfer cascade unavailable: {type(exc).__name__}: {exc}")
        return None


CASCADE_CONFIGS = [
    # (name, group sizes, prefix lens, own lens) with Llama-3-8B heads (32/8/128), page 16, bf16
    ("cascade_b64_prefix4096_own512", [64], [4096], [512] * 64),
    ("cascade_8x8_prefix2048_own256", [8] * 8, [2048] * 8, [256] * 64),
]


@pytest.mark.parametrize("name,groups,plens,lens", CASCADE_CONFIGS)
def test_cascade_against_flashinfer_on_the_same_gpu(name, groups, plens, lens):
    """Shared-prefix decode: this repository's one-launch cascade, the same problem without
    sharing through its plain decode, FlashInfer's two-level cascade and FlashInfer's plain decode.
    Bytes are the unique KV bytes (each prefix once) plus q and out."""
    from kernel_lab import cuda_ops
    from kernel_lab.kv_cache import random_cascade_problem

    q, kv = random_cascade_problem(groups, plens, lens, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=5)
    table, clens = kv.concatenated_tables()
    args = (kv.k_cache, kv.v_cache, kv.prefix_block_table, kv.prefix_lens, kv.prefix_indptr, kv.block_table,
            kv.seq_lens)
    ours = cuda_ops.paged_decode_attention_cascade(q, *args)
    unique = (sum(plens) + sum(lens)) * 8 * 128 * 2 * 2 + 2 * len(lens) * 32 * 128 * 2
    times = {
        "b200_cascade": device_us(lambda: cuda_ops.paged_decode_attention_cascade(q, *args), 50),
        "b200_plain_concat": device_us(
            lambda: cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, table, clens), 50),
    }
    fi = flashinfer_cascade(q, kv)
    if fi is not None:
        run, fi_out = fi
        torch.cuda.synchronize()
        torch.testing.assert_close(fi_out, ours, **tolerance(torch.bfloat16))
        times["flashinfer_cascade"] = device_us(run, 30)
    ctx = max(clens.tolist())
    if all(n == ctx for n in clens.tolist()):
        plain = type("KV", (), {"k_cache": kv.k_cache, "v_cache": kv.v_cache, "block_table": table})()
        fi2 = flashinfer_decode(q, plain, ctx)
        if fi2 is not None:
            times["flashinfer_plain_concat"] = device_us(fi2[0], 30)
    _report(name, unique, times)
