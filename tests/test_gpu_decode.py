"""Paged decode attention on the GPU vs the oracle and the reference's golden vectors.

Calls go through the C ABI (``kernel_lab.capi`` -> libkernel_lab_b200.so) and through the
drop-in torch op (``kernel_lab.cuda_ops``). Tolerances: kernel-lab's per-dtype table
(fp32 1e-4, fp16 2e-3, bf16 1.6e-2) against the golden vectors, and the north star's
max-abs bound (fp16 2e-3, bf16 2e-2) against the fp32-math oracle. Spare pages are
NaN-poisoned throughout, so any read of a page outside the block table fails the test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import (
    DT,
    DT_NAME,
    NORTH_STAR_MAX_ABS,
    assert_within_abs_or_ulp,
    build_decode_case,
    golden_array,
    golden_index,
    golden_to_torch,
    tolerance,
    to_f32_numpy,
)

pytestmark = pytest.mark.gpu

DECODE_CASES = [c["name"] for c in golden_index()["decode"]]


def run_capi(q, kv, scale=None, num_splits=0):
    from kernel_lab import capi

    out = torch.full_like(q, float("nan"))
    scratch = capi.paged_decode(out, q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, scale, num_splits)
    torch.cuda.synchronize()
    assert scratch.status() == 0
    return out


def run_op(q, kv, scale=None, num_splits=None):
    from kernel_lab import cuda_ops

    return cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, scale, num_splits)


def oracle_out(q, kv, scale=None):
    """The oracle on the pages the block table actually names (gathered on the device first,
    so a multi-gigabyte pool is not copied to the host)."""
    lens = kv.seq_lens.cpu()
    page = kv.page_size
    need = [(max(int(n), 0) + page - 1) // page for n in lens]
    width = max(max(need), 1)
    ids = torch.cat([kv.block_table[b, :n].long() for b, n in enumerate(need)] + [torch.zeros(0, dtype=torch.long, device=kv.block_table.device)])
    table = np.zeros((len(need), width), np.int32)
    cur = 0
    for b, n in enumerate(need):
        table[b, :n] = np.arange(cur, cur + n)
        cur += n
    k = kv.k_cache[ids] if ids.numel() else kv.k_cache[:1]
    v = kv.v_cache[ids] if ids.numel() else kv.v_cache[:1]
    return oracle.paged_decode_attention(
        to_f32_numpy(q), to_f32_numpy(k), to_f32_numpy(v), table, lens.numpy(), scale, "f32",
    )


def assert_close_to_oracle(got, want_f32, dtype):
    """North-star bound (fp16 2e-3, bf16 2e-2 max-abs) against the unrounded fp32 oracle, or
    one storage ulp where the output is large enough that one ulp exceeds it."""
    assert NORTH_STAR_MAX_ABS[dtype] > 0
    assert_within_abs_or_ulp(got, want_f32, dtype)


@pytest.mark.parametrize("name", DECODE_CASES)
def test_golden_cases_through_c_abi(name):
    case = next(c for c in golden_index()["decode"] if c["name"] == name)
    q, kv, _, _ = build_decode_case(case, device="cuda")
    got = run_capi(q, kv, case.get("scale"))
    want = golden_to_torch(golden_array("decode", f"{name}/out"), case["dt"]).cuda()
    torch.testing.assert_close(got, want, **tolerance(DT[case["dt"]]))
    assert_close_to_oracle(got, oracle_out(q, kv, case.get("scale")), DT[case["dt"]])


@pytest.mark.parametrize("name", ["cfg1", "cu_32_8_128_bf16", "cfg4_32_1", "cfg4_32_32", "tri_8_2_f32"])
def test_golden_cases_through_torch_op(name):
    case = next(c for c in golden_index()["decode"] if c["name"] == name)
    q, kv, _, _ = build_decode_case(case, device="cuda")
    got = run_op(q, kv, case.get("scale"))
    want = golden_to_torch(golden_array("decode", f"{name}/out"), case["dt"]).cuda()
    torch.testing.assert_close(got, want, **tolerance(DT[case["dt"]]))
    from kernel_lab import cuda_ops

    assert cuda_ops.decode_status(clear=True) == 0


def test_reference_signature_entry_point():
    """kl_paged_decode_attention takes exactly kernel-lab's launcher arguments."""
    from kernel_lab import capi

    case = next(c for c in golden_index()["decode"] if c["name"] == "cu_16_4_128_f16")
    q, kv, _, _ = build_decode_case(case, device="cuda")
    out = torch.full_like(q, float("nan"))
    capi.paged_decode_attention(out, q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens)
    want = golden_to_torch(golden_array("decode", "cu_16_4_128_f16/out"), "f16").cuda()
    torch.testing.assert_close(out, want, **tolerance(torch.float16))


@pytest.mark.parametrize("num_splits", [1, 2, 3, 5, 7, 16, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_split_count_never_changes_the_result(num_splits, dtype):
    """Splits only re-partition the sum (kernel-lab tests/test_paged_attention.py:32-37); many
    splits leave some empty, which the merge must weight at zero."""
    from kernel_lab.kv_cache import random_decode_problem

    lens = [1, 15, 16, 17, 33, 70]
    head_dim = 32 if dtype == torch.float32 else 128
    q, kv, _, _ = random_decode_problem(lens, 4, 2, head_dim, 16, dtype=dtype, device="cuda")
    got = run_capi(q, kv, num_splits=num_splits)
    want = oracle_out(q, kv)
    if dtype == torch.float32:
        np.testing.assert_allclose(got.cpu().numpy(), want, atol=1e-5, rtol=1e-5)
    else:
        assert_close_to_oracle(got, want, dtype)
        auto = run_capi(q, kv)
        torch.testing.assert_close(got, auto, atol=2e-2, rtol=0)


@pytest.mark.parametrize("num_splits", [1, 4, 32, 64])
def test_split_sweep_on_config3_geometry(num_splits):
    """Config 3 geometry (32/8/128 bf16, page 16) at batch 8, context 512, splits 1..64
    (64 splits of 32 pages leave 32 splits empty)."""
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([512] * 8, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda")
    got = run_capi(q, kv, num_splits=num_splits)
    want = golden_to_torch(golden_array("decode", "cfg3_b8_512/out"), "bf16").cuda()
    torch.testing.assert_close(got, want, **tolerance(torch.bfloat16))


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 4), (8, 1), (32, 8), (32, 1), (64, 8), (12, 3), (48, 2)])
@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_head_layouts(hq, hkv, head_dim, dtype):
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([1, 3, 16, 17, 300, 1025], hq, hkv, head_dim, 16, dtype=dtype, device="cuda")
    assert_close_to_oracle(run_capi(q, kv), oracle_out(q, kv), dtype)


@pytest.mark.parametrize(
    "hq,hkv,head_dim,nt",
    [
        (48, 2, 128, "2"),  # 16 query heads a warp (KL_DECODE_NT=2): two KV heads a tile, two
        (64, 2, 128, "2"),  # query groups a head, two warps splitting each (head, group)'s tiles
        (32, 2, 256, "0"),  # head_dim 256: 8 heads a warp, the same tile shape
        (32, 2, 128, "1"),  # 8 query heads a warp (the default at this size) on groups of 16 and 12
        (24, 2, 128, "0"),
        (64, 4, 128, "1"),  # four heads a tile, two groups, no split warps
    ],
)
def test_tiles_of_several_heads_and_query_groups(hq, hkv, head_dim, nt, monkeypatch):
    """Enough tiles that a tile holds two or more KV heads and each head's query heads span two
    warp groups. The warps that split a (head, group)'s tiles combine through shared memory, and
    the combine must find each partner warp's slot in the warp-index order: a mix-up of (head,
    group) orders there only shows when both counts exceed one."""
    from kernel_lab.kv_cache import random_decode_problem

    monkeypatch.setenv("KL_DECODE_NT", nt)
    q, kv, _, _ = random_decode_problem([1024] * 16 + [3000, 17], hq, hkv, head_dim, 16, dtype=torch.bfloat16,
                                        device="cuda")
    assert_close_to_oracle(run_capi(q, kv), oracle_out(q, kv), torch.bfloat16)


@pytest.mark.parametrize("page_size", [1, 4, 8, 16, 32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_page_sizes(page_size, dtype):
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([3, 50, 129, 250], 8, 2, 128, page_size, dtype=dtype, device="cuda")
    got = run_capi(q, kv)
    if dtype == torch.float32:
        np.testing.assert_allclose(got.cpu().numpy(), oracle_out(q, kv), atol=1e-4, rtol=1e-4)
    else:
        assert_close_to_oracle(got, oracle_out(q, kv), dtype)


def test_one_hot_known_answer():
    """One key far more aligned than the rest and v[t] = t gives exactly 13.0
    (kernel-lab tests/test_paged_attention.py:81-91), on both kernels."""
    from kernel_lab.kv_cache import build_paged_kv

    for dtype, d in ((torch.float32, 32), (torch.bfloat16, 128), (torch.float16, 64)):
        keys = [torch.zeros(20, 1, d, dtype=dtype)]
        values = [torch.arange(20, dtype=torch.float32)[:, None, None].expand(20, 1, d).to(dtype)]
        keys[0][13, 0, 0] = 100.0
        kv = build_paged_kv([k.cuda() for k in keys], [v.cuda() for v in values], page_size=16)
        q = torch.zeros(1, 1, d, device="cuda", dtype=dtype)
        q[0, 0, 0] = 1.0
        out = run_capi(q, kv, scale=1.0)
        torch.testing.assert_close(out.float(), torch.full_like(out.float(), 13.0), atol=1e-4, rtol=0)


def test_poisoned_pages_and_padding_are_never_read():
    """NaN spare pages, NaN block-table padding target and NaN tails of partial pages: the
    result must stay finite and exact (stricter than kernel-lab's 1e4 poison)."""
    from kernel_lab.kv_cache import random_decode_problem

    for dtype, d in ((torch.bfloat16, 128), (torch.float32, 32)):
        q, kv, _, _ = random_decode_problem([20, 9, 33], 8, 2, d, 16, dtype=dtype, device="cuda")
        want = oracle_out(q, kv)
        # Poison the unused tail of every partially filled page as well.
        for b, n in enumerate(kv.seq_lens.tolist()):
            last = int(kv.block_table[b, (n - 1) // 16])
            kv.k_cache[last, n % 16 or 16 :] = float("nan")
            kv.v_cache[last, n % 16 or 16 :] = float("nan")
        got = run_capi(q, kv)
        assert torch.isfinite(got).all()
        assert_close_to_oracle(got, want, dtype)


def test_custom_scale_and_padded_block_table():
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([5, 20, 64], 4, 2, 128, 16, dtype=torch.bfloat16, device="cuda")
    kv.block_table = torch.nn.functional.pad(kv.block_table, (0, 6))  # extra columns (page 0 = maybe poisoned)
    for scale in (0.05, 1.0):
        assert_close_to_oracle(run_capi(q, kv, scale=scale), oracle_out(q, kv, scale), torch.bfloat16)


def test_zero_length_sequences_give_zeros():
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([5, 40, 3], 8, 2, 128, 16, dtype=torch.bfloat16, device="cuda")
    kv.seq_lens[1] = 0
    for splits in (0, 3):
        got = run_capi(q, kv, num_splits=splits)
        assert (got[1] == 0).all()
        assert_close_to_oracle(got, oracle_out(q, kv), torch.bfloat16)


def test_bad_page_ids_are_flagged_not_followed():
    from kernel_lab import capi
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([40, 40], 8, 2, 128, 16, dtype=torch.bfloat16, device="cuda")
    kv.block_table[1, 1] = kv.k_cache.shape[0] + 100  # outside the pool
    out = torch.empty_like(q)
    scratch = capi.paged_decode(out, q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens)
    torch.cuda.synchronize()
    assert scratch.status(clear=True) & capi.KL_STATUS_BAD_PAGE
    assert scratch.status() == 0
    good = oracle_out(q[:1], type(kv)(kv.k_cache, kv.v_cache, kv.block_table[:1], kv.seq_lens[:1], 16))
    assert_close_to_oracle(out[:1], good, torch.bfloat16)


def test_scratch_is_reusable_across_shapes():
    """One scratch pair serves successive calls of different batch sizes (counters self-reset)."""
    from kernel_lab import capi
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([700] * 16, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda")
    scratch = capi.DecodeScratch.for_problem(q, kv.k_cache, kv.block_table)
    for lens in ([700] * 16, [5, 900, 31], [300] * 16, [1000, 1, 1, 2]):
        qq, kk, _, _ = random_decode_problem(lens, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=len(lens))
        out = torch.empty_like(qq)
        capi.paged_decode(out, qq, kk.k_cache, kk.v_cache, kk.block_table, kk.seq_lens, scratch=scratch)
        torch.cuda.synchronize()
        assert_close_to_oracle(out, oracle_out(qq, kk), torch.bfloat16)
    assert scratch.status() == 0
    assert int(scratch.sync[4:].view(torch.int32).abs().sum()) == 0


@pytest.mark.parametrize("hq,hkv", [(32, 1), (32, 8), (32, 32)])
def test_ragged_batch_config4_sample(hq, hkv):
    """Config 4's ragged lengths (uniform in [1, 32768], with 16k-1, 16k, 16k+1) at batch 16;
    three sequences are checked against the oracle in full."""
    from kernel_lab.kv_cache import random_paged_pool

    rng = np.random.default_rng(4)
    lens = [16383, 16384, 16385, 1, 15, 16, 17] + rng.integers(1, 32769, size=9).tolist()
    q, kv = random_paged_pool(lens, hq, hkv, 128, 16, dtype=torch.bfloat16, device="cuda", seed=4)
    got = run_capi(q, kv)
    for b in (0, 3, 10):
        sub = type(kv)(kv.k_cache, kv.v_cache, kv.block_table[b : b + 1], kv.seq_lens[b : b + 1], 16)
        assert_close_to_oracle(got[b : b + 1], oracle_out(q[b : b + 1], sub), torch.bfloat16)
    forced = run_capi(q, kv, num_splits=64)
    torch.testing.assert_close(got, forced, atol=2e-2, rtol=0)


def test_full_size_headline_properties():
    """Config 3 headline (batch 64, context 4096, 32/8/128 bf16) at full size, checked by
    size-independent properties: planner == forced single split (a different partition),
    invariance under a page permutation of the pool, linearity in V, and an oracle check
    of two complete sequences."""
    from kernel_lab.kv_cache import random_paged_pool

    q, kv = random_paged_pool([4096] * 64, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=3)
    got = run_capi(q, kv)
    torch.testing.assert_close(got, run_capi(q, kv, num_splits=1), atol=2e-2, rtol=0)
    torch.testing.assert_close(got, run_op(q, kv), atol=0, rtol=0)  # deterministic

    perm = torch.randperm(kv.k_cache.shape[0], device="cuda")
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device="cuda")
    moved = type(kv)(kv.k_cache[perm], kv.v_cache[perm], inv[kv.block_table.long()].int(), kv.seq_lens, 16)
    torch.testing.assert_close(run_capi(q, moved), got, atol=0, rtol=0)

    # Linearity in V: attn(V1 + V2) ~= attn(V1) + attn(V2) (same K, so the same softmax).
    v2 = torch.randn_like(kv.v_cache, dtype=torch.float32).to(torch.bfloat16)
    kv2 = type(kv)(kv.k_cache, v2, kv.block_table, kv.seq_lens, 16)
    vs = (kv.v_cache.float() + v2.float()).to(torch.bfloat16)
    kv_sum = type(kv)(kv.k_cache, vs, kv.block_table, kv.seq_lens, 16)
    lhs = run_capi(q, kv_sum).float()
    rhs = got.float() + run_capi(q, kv2).float()
    assert (lhs - rhs).abs().max().item() < 4e-2

    for b in (0, 63):
        sub = type(kv)(kv.k_cache, kv.v_cache, kv.block_table[b : b + 1], kv.seq_lens[b : b + 1], 16)
        assert_close_to_oracle(got[b : b + 1], oracle_out(q[b : b + 1], sub), torch.bfloat16)


def test_ops_work_under_torch_compile():
    """kernel-lab tests/test_cuda_kernels.py:56-66, for both op families."""
    from kernel_lab import cuda_ops  # noqa: F401
    from kernel_lab.kv_cache import random_decode_problem

    x = torch.randn(4, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(256, device="cuda", dtype=torch.float16)

    @torch.compile(fullgraph=True)
    def f(x, w):
        out = torch.empty_like(x)
        torch.ops.kernel_lab.rms_norm(out, x, w, 1e-6)
        return out * 2

    want = oracle.rms_norm(to_f32_numpy(x), to_f32_numpy(w), 1e-6, "f16") * 2
    np.testing.assert_allclose(f(x, w).float().cpu().numpy(), want, atol=4e-3, rtol=4e-3)

    q, kv, _, _ = random_decode_problem([7, 100], 8, 2, 128, 16, dtype=torch.bfloat16, device="cuda")

    @torch.compile(fullgraph=True)
    def g(q, k, v, bt, ln):
        out = torch.empty_like(q)
        torch.ops.kernel_lab.paged_decode_attention(out, q, k, v, bt, ln, 128**-0.5)
        return out + 1

    got = g(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens) - 1
    assert_close_to_oracle(got, oracle_out(q, kv), torch.bfloat16)


def test_validation_errors_are_runtime_errors():
    from kernel_lab import cuda_ops
    from kernel_lab.kv_cache import random_decode_problem

    q, kv, _, _ = random_decode_problem([4], 3, 2, 32, 16, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="multiple"):
        cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens)
    q, kv, _, _ = random_decode_problem([4], 2, 2, 32, 16, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="int32"):
        cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table.long(), kv.seq_lens)
    assert DT_NAME[q.dtype] == "f32"
