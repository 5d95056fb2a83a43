"""Paged KV append on the GPU (the write side of the paged cache).

The kernel is a copy, so it must equal the append oracle bit for bit: every dtype, positions on
and across page boundaries, padding sequences (negative positions), rows taken as strided views
of a fused QKV projection, and bad page ids (skipped, reported in the status word). The round
trip ties it to the read side: appending the last token of every sequence into a pool that
holds the others, then decoding, gives exactly what decoding the complete pool gives.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import DT

pytestmark = pytest.mark.gpu


def _pool(lens, hkv, d, page, dtype, seed=0):
    from kernel_lab.kv_cache import random_paged_pool

    return random_paged_pool(lens, 4 * hkv, hkv, d, page, dtype=dtype, device="cuda", seed=seed)


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("via", ["capi", "op"])
def test_append_matches_the_oracle_bit_for_bit(dtype, via):
    from kernel_lab import capi, cuda_ops

    dt = DT[dtype]
    lens = [1, 15, 16, 17, 63, 64, 200, 5]
    _, kv = _pool(lens, 4, 128, 16, dt, seed=2)
    g = torch.Generator(device="cuda").manual_seed(9)
    k_new = torch.randn(len(lens), 4, 128, generator=g, device="cuda").to(dt)
    v_new = torch.randn(len(lens), 4, 128, generator=g, device="cuda").to(dt)
    # Each sequence's last allocated token (first and last slots of pages among them), and a skip.
    pos = torch.tensor([0, 14, 15, 16, 62, 63, 199, -1], dtype=torch.int32, device="cuda")
    want_k, want_v, want_status = oracle.paged_kv_append(
        _f32(kv.k_cache), _f32(kv.v_cache), _f32(k_new), _f32(v_new), kv.block_table.cpu().numpy(), pos.cpu().numpy()
    )
    if via == "capi":
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        capi.paged_kv_append(kv.k_cache, kv.v_cache, k_new, v_new, kv.block_table, pos, status=status)
        got_status = int(status.item())
    else:
        cuda_ops.decode_status(clear=True)
        cuda_ops.paged_kv_append(kv.k_cache, kv.v_cache, k_new, v_new, kv.block_table, pos)
        got_status = cuda_ops.decode_status(clear=True)
    torch.cuda.synchronize()
    assert got_status == want_status == 0
    np.testing.assert_array_equal(_f32(kv.k_cache), want_k)  # NaN spares compare equal in place
    np.testing.assert_array_equal(_f32(kv.v_cache), want_v)


def test_append_from_a_fused_qkv_view_and_odd_head_dim():
    from kernel_lab import cuda_ops

    lens = [3, 33, 100]
    hq, hkv, d = 8, 2, 128
    _, kv = _pool(lens, hkv, d, 16, torch.bfloat16, seed=4)
    qkv = torch.randn(len(lens), (hq + 2 * hkv) * d, device="cuda").to(torch.bfloat16)
    k_view = qkv[:, hq * d : (hq + hkv) * d].view(len(lens), hkv, d)  # rows (hq + 2 hkv) * d apart
    v_view = qkv[:, (hq + hkv) * d :].view(len(lens), hkv, d)
    pos = torch.tensor([3, 32, 99], dtype=torch.int32, device="cuda")
    want_k, want_v, _ = oracle.paged_kv_append(
        _f32(kv.k_cache), _f32(kv.v_cache), _f32(k_view), _f32(v_view), kv.block_table.cpu().numpy(), pos.cpu().numpy()
    )
    cuda_ops.paged_kv_append(kv.k_cache, kv.v_cache, k_view, v_view, kv.block_table, pos)
    np.testing.assert_array_equal(_f32(kv.k_cache), want_k)
    np.testing.assert_array_equal(_f32(kv.v_cache), want_v)

    # head_dim 36 (rows of 72 bytes): the element path.
    _, kv2 = _pool([5, 20], 2, 36, 8, torch.float16, seed=6)
    kn = torch.randn(2, 2, 36, device="cuda").half()
    pos2 = torch.tensor([5, 19], dtype=torch.int32, device="cuda")
    want_k2, _, _ = oracle.paged_kv_append(
        _f32(kv2.k_cache), _f32(kv2.v_cache), _f32(kn), _f32(kn), kv2.block_table.cpu().numpy(), pos2.cpu().numpy()
    )
    cuda_ops.paged_kv_append(kv2.k_cache, kv2.v_cache, kn, kn, kv2.block_table, pos2)
    np.testing.assert_array_equal(_f32(kv2.k_cache), want_k2)


def test_bad_pages_and_positions_are_skipped_and_flagged():
    from kernel_lab import cuda_ops

    _, kv = _pool([16, 16], 2, 64, 16, torch.float16, seed=8)
    before_k = kv.k_cache.clone()
    bt = kv.block_table.clone()
    bt[0, 0] = kv.k_cache.shape[0] + 3  # page id past the pool
    kn = torch.ones(2, 2, 64, device="cuda").half()
    pos = torch.tensor([0, 16 * bt.shape[1]], dtype=torch.int32, device="cuda")  # 2nd: past the table
    cuda_ops.decode_status(clear=True)
    cuda_ops.paged_kv_append(kv.k_cache, kv.v_cache, kn, kn, bt, pos)
    assert cuda_ops.decode_status(clear=True) & 1
    assert torch.equal(kv.k_cache.view(torch.int16), before_k.view(torch.int16))  # nothing written


@pytest.mark.parametrize("hq,hkv", [(32, 8), (64, 8), (32, 32)])
def test_append_then_decode_equals_decode_of_the_complete_pool(hq, hkv):
    """Decode step of a serving loop: the pool holds tokens [0, len-1) of every sequence; the new
    token's K/V are appended at position len-1 and the decode over len tokens must equal the
    decode of the pool that was built with all len tokens."""
    from kernel_lab import cuda_ops
    from kernel_lab.kv_cache import random_paged_pool

    lens = [1, 16, 17, 300, 1024, 4095]
    q, full = random_paged_pool(lens, hq, hkv, 128, 16, dtype=torch.bfloat16, device="cuda", seed=12)
    last = torch.tensor(lens, dtype=torch.int32, device="cuda") - 1
    rows = torch.arange(len(lens), device="cuda")
    pages = full.block_table[rows, (last // 16).long()].long()
    slots = (last % 16).long()
    k_new = full.k_cache[pages, slots].clone()
    v_new = full.v_cache[pages, slots].clone()
    want = cuda_ops.paged_decode_attention(q, full.k_cache, full.v_cache, full.block_table, full.seq_lens)
    # Remove the last token (poison its slot), append it back, decode again.
    full.k_cache[pages, slots] = float("nan")
    full.v_cache[pages, slots] = float("nan")
    cuda_ops.paged_kv_append(full.k_cache, full.v_cache, k_new, v_new, full.block_table, last)
    got = cuda_ops.paged_decode_attention(q, full.k_cache, full.v_cache, full.block_table, full.seq_lens)
    assert cuda_ops.decode_status(clear=True) == 0
    assert torch.equal(got, want)
