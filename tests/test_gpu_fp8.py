"""FP8 (e4m3) KV cache on the GPU: decode against the oracle, quantising append, round trips.

The cache holds e4m3 codes with one float32 scale per KV head (kernel-lab's roadmap item,
README.md:98). The decode's reference is the oracle's fp32 attention over the dequantised cache
(code value * scale), so the bound is the north star's: max-abs 2e-3 (fp16) / 2e-2 (bf16), or one
storage ulp where the output is large. The append is a quantiser and must equal the oracle's
e4m3(x / scale) bit for bit. Spare pages are poisoned with NaN codes and never read.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import assert_within_abs_or_ulp

pytestmark = pytest.mark.gpu


def _fp8_problem(lens, hq, hkv, d, page, dtype, seed=0):
    from kernel_lab.kv_cache import e4m3_scales, quantize_e4m3, random_paged_pool

    q, kv = random_paged_pool(lens, hq, hkv, d, page, dtype=dtype, device="cuda", seed=seed)
    ks, vs = e4m3_scales(kv.k_cache), e4m3_scales(kv.v_cache)
    return q, kv, quantize_e4m3(kv.k_cache, ks), quantize_e4m3(kv.v_cache, vs), ks, vs


def _oracle(q, kv, k8, v8, ks, vs, scale=None):
    """The oracle on the pages the block table names (gathered first: pools can be large)."""
    lens = kv.seq_lens.cpu()
    page = kv.page_size
    need = [(max(int(n), 0) + page - 1) // page for n in lens]
    ids = torch.cat([kv.block_table[b, :n].long() for b, n in enumerate(need)])
    table = np.zeros((len(need), max(max(need), 1)), np.int32)
    cur = 0
    for b, n in enumerate(need):
        table[b, :n] = np.arange(cur, cur + n)
        cur += n
    return oracle.paged_decode_attention_fp8(
        q.float().cpu().numpy(), k8[ids].view(torch.uint8).cpu().numpy(), v8[ids].view(torch.uint8).cpu().numpy(),
        ks.cpu().numpy(), vs.cpu().numpy(), table, lens.numpy(), scale, "f32",
    )


CASES = [
    # (lens, hq, hkv, d, page)
    ([1, 15, 16, 17, 33, 70], 32, 8, 128, 16),
    ([1, 3, 16, 17, 300, 1025], 64, 8, 128, 16),
    ([5, 100, 513], 32, 32, 128, 16),
    ([7, 64, 200], 16, 4, 128, 8),
    ([9, 250], 32, 8, 256, 16),
    ([2000, 17], 32, 1, 128, 32),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_decode_matches_the_oracle(case, dtype):
    from kernel_lab import cuda_ops

    lens, hq, hkv, d, page = CASES[case]
    q, kv, k8, v8, ks, vs = _fp8_problem(lens, hq, hkv, d, page, dtype, seed=case)
    cuda_ops.decode_status(clear=True)
    got = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv.block_table, kv.seq_lens)
    assert cuda_ops.decode_status(clear=True) == 0
    assert_within_abs_or_ulp(got, _oracle(q, kv, k8, v8, ks, vs), dtype)


def test_fp8_decode_is_close_to_the_16_bit_decode_it_quantises():
    """e4m3 keeps 3 mantissa bits: the output of attention over the quantised cache stays
    within a few percent of the bf16 cache's (attention averages the per-element errors)."""
    from kernel_lab import cuda_ops

    q, kv, k8, v8, ks, vs = _fp8_problem([300, 1025, 4096], 32, 8, 128, 16, torch.bfloat16, seed=3)
    ref = cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens)
    got = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv.block_table, kv.seq_lens)
    err = (got.float() - ref.float()).abs().max().item()
    assert err < 0.1 * ref.float().abs().max().item(), err


def test_fp8_forced_splits_and_capi_agree_with_the_planner():
    from kernel_lab import capi, cuda_ops

    q, kv, k8, v8, ks, vs = _fp8_problem([700] * 16, 32, 8, 128, 16, torch.bfloat16, seed=5)
    want = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv.block_table, kv.seq_lens)
    for splits in (0, 1, 3, 64):
        out = torch.full_like(q, float("nan"))
        scratch = capi.paged_decode_fp8(out, q, k8, v8, ks, vs, kv.block_table, kv.seq_lens, num_splits=splits)
        torch.cuda.synchronize()
        assert scratch.status() == 0
        if splits == 0:
            assert torch.equal(out, want)
        torch.testing.assert_close(out, want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_fp8_append_quantises_like_the_oracle(dtype):
    from kernel_lab import cuda_ops

    lens = [1, 15, 16, 17, 63, 200]
    q, kv, k8, v8, ks, vs = _fp8_problem(lens, 16, 4, 128, 16, torch.bfloat16, seed=9)
    g = torch.Generator(device="cuda").manual_seed(1)
    k_new = (torch.randn(len(lens), 4, 128, generator=g, device="cuda") * 3).to(dtype)
    v_new = (torch.randn(len(lens), 4, 128, generator=g, device="cuda") * 3).to(dtype)
    k_new[0, 0, 0] = 1e5  # saturates
    pos = torch.tensor([0, 14, 15, 16, 62, -1], dtype=torch.int32, device="cuda")
    want_k, want_v, _ = oracle.paged_kv_append_fp8(
        k8.view(torch.uint8).cpu().numpy(), v8.view(torch.uint8).cpu().numpy(), k_new.float().cpu().numpy(),
        v_new.float().cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy(), kv.block_table.cpu().numpy(),
        pos.cpu().numpy(),
    )
    cuda_ops.decode_status(clear=True)
    cuda_ops.paged_kv_append_fp8(k8, v8, k_new, v_new, ks, vs, kv.block_table, pos)
    assert cuda_ops.decode_status(clear=True) == 0
    np.testing.assert_array_equal(k8.view(torch.uint8).cpu().numpy(), want_k)
    np.testing.assert_array_equal(v8.view(torch.uint8).cpu().numpy(), want_v)


def test_fp8_append_then_decode_equals_decode_of_the_quantised_pool():
    from kernel_lab import cuda_ops
    from kernel_lab.kv_cache import random_paged_pool

    lens = [1, 16, 17, 300, 4095]
    q, full, k8, v8, ks, vs = _fp8_problem(lens, 32, 8, 128, 16, torch.bfloat16, seed=12)
    want = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, full.block_table, full.seq_lens)
    last = torch.tensor(lens, dtype=torch.int32, device="cuda") - 1
    rows = torch.arange(len(lens), device="cuda")
    pages = full.block_table[rows, (last // 16).long()].long()
    slots = (last % 16).long()
    k_new = full.k_cache[pages, slots].clone()  # the bf16 rows the pool was quantised from
    v_new = full.v_cache[pages, slots].clone()
    k8.view(torch.uint8)[pages, slots] = 0x7F  # NaN codes where the last token was
    v8.view(torch.uint8)[pages, slots] = 0x7F
    cuda_ops.paged_kv_append_fp8(k8, v8, k_new, v_new, ks, vs, full.block_table, last)
    got = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, full.block_table, full.seq_lens)
    assert cuda_ops.decode_status(clear=True) == 0
    assert torch.equal(got, want)


def test_fp8_headline_size_is_deterministic_and_matches_two_full_sequences():
    from kernel_lab import cuda_ops

    q, kv, k8, v8, ks, vs = _fp8_problem([4096] * 64, 32, 8, 128, 16, torch.bfloat16, seed=13)
    a = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv.block_table, kv.seq_lens)
    b = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv.block_table, kv.seq_lens)
    assert torch.equal(a, b) and cuda_ops.decode_status(clear=True) == 0
    for i in (0, 37):
        sub = type(kv)(kv.k_cache, kv.v_cache, kv.block_table[i : i + 1], kv.seq_lens[i : i + 1], 16)
        assert_within_abs_or_ulp(a[i : i + 1], _oracle(q[i : i + 1], sub, k8, v8, ks, vs), torch.bfloat16)


def test_fp8_rejects_unsupported_shapes():
    from kernel_lab import cuda_ops

    q, kv, k8, v8, ks, vs = _fp8_problem([20], 8, 2, 64, 16, torch.bfloat16)
    with pytest.raises(RuntimeError):
        cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv.block_table, kv.seq_lens)
