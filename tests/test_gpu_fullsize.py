"""Every sequence of the benchmark configurations against the fp32 oracle, at full size.

kernel-lab's own long-context check compares its kernel with the reference on whole sequences
(tests/test_paged_attention.py:103-106 there); here every sequence of each benchmark-sized
problem is compared, at the north star's bound (max-abs 2e-2 for bf16 against the unrounded fp32
oracle, or one bf16 ulp where the output is large enough that one ulp exceeds it):

* config 3's headline: batch 64 x context 4096, Llama-3-8B heads 32/8/128 (also over an e4m3
  cache with per-KV-head scales);
* config 5: batch 256 x context 8192, Llama-3-70B heads 64/8/128 (8.6 GB of KV);
* config 4: batch 128, lengths uniform in [1, 32768] plus 16k - 1, 16k and 16k + 1, in the MQA
  (32/1), GQA (32/8) and MHA (32/32) layouts (up to 37 GB of KV).

Each sequence's pages are gathered on the GPU and widened to fp32 there (an exact conversion),
copied to the host, and the NumPy oracle runs on host threads (NumPy releases the interpreter
lock inside its kernels), a bounded number of sequences in flight.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import assert_within_abs_or_ulp

pytestmark = pytest.mark.gpu

THREADS = 8


def oracle_every_sequence(q, kv, scale=None, fp8_scales=None) -> np.ndarray:
    """The fp32 oracle's output [batch, Hq, D] for every sequence of `kv` (an e4m3 cache when
    fp8_scales = (k_scale, v_scale) is given)."""
    lens = kv.seq_lens.cpu().tolist()
    page = kv.page_size
    qf = q.float().cpu().numpy()
    out = np.zeros(qf.shape, np.float32)
    if fp8_scales is not None:
        ks, vs = (s.cpu().numpy() for s in fp8_scales)

    def one(b, kb, vb, n):
        table = np.arange(kb.shape[0], dtype=np.int32)[None]
        if fp8_scales is None:
            out[b] = oracle.paged_decode_attention(qf[b : b + 1], kb, vb, table, np.array([n]), scale, "f32")[0]
        else:
            out[b] = oracle.paged_decode_attention_fp8(qf[b : b + 1], kb, vb, ks, vs, table, np.array([n]), scale,
                                                       "f32")[0]

    with ThreadPoolExecutor(THREADS) as pool:
        pending = []
        for b, n in enumerate(lens):
            if n <= 0:
                continue
            ids = kv.block_table[b, : (n + page - 1) // page].long()
            if fp8_scales is None:
                kb, vb = kv.k_cache[ids].float().cpu().numpy(), kv.v_cache[ids].float().cpu().numpy()
            else:
                kb = kv.k_cache[ids].view(torch.uint8).cpu().numpy()
                vb = kv.v_cache[ids].view(torch.uint8).cpu().numpy()
            pending.append(pool.submit(one, b, kb, vb, n))
            if len(pending) >= THREADS:
                pending.pop(0).result()
        for f in pending:
            f.result()
    return out


def _decode(q, kv):
    from kernel_lab import capi

    out = torch.full_like(q, float("nan"))
    scratch = capi.paged_decode(out, q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens)
    torch.cuda.synchronize()
    assert scratch.status() == 0
    return out


def test_headline_every_sequence_matches_the_oracle():
    """Config 3's headline, batch 64 x 4096, 32/8/128 bf16: all 64 sequences, through the C ABI
    and through the torch op (bit-identical: one deterministic kernel)."""
    from kernel_lab import cuda_ops
    from kernel_lab.kv_cache import random_paged_pool

    q, kv = random_paged_pool([4096] * 64, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=3)
    got = _decode(q, kv)
    assert torch.equal(got, cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens))
    assert_within_abs_or_ulp(got, oracle_every_sequence(q, kv), torch.bfloat16)


def test_headline_e4m3_cache_every_sequence_matches_the_oracle():
    """The headline over an e4m3 cache with per-KV-head scales: all 64 sequences against the
    oracle's attention over the dequantised cache."""
    from kernel_lab import cuda_ops
    from kernel_lab.kv_cache import e4m3_scales, quantize_e4m3, random_paged_pool

    q, kv = random_paged_pool([4096] * 64, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=13)
    ks, vs = e4m3_scales(kv.k_cache), e4m3_scales(kv.v_cache)
    k8, v8 = quantize_e4m3(kv.k_cache, ks), quantize_e4m3(kv.v_cache, vs)
    kv8 = type(kv)(k8, v8, kv.block_table, kv.seq_lens, kv.page_size)
    del kv
    got = cuda_ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, kv8.block_table, kv8.seq_lens)
    assert cuda_ops.decode_status(clear=True) == 0
    assert_within_abs_or_ulp(got, oracle_every_sequence(q, kv8, fp8_scales=(ks, vs)), torch.bfloat16)


def test_config5_every_sequence_matches_the_oracle():
    """Config 5's geometry on one GPU: batch 256 x context 8192, Llama-3-70B heads 64/8/128."""
    from kernel_lab.kv_cache import random_paged_pool

    q, kv = random_paged_pool([8192] * 256, 64, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=5)
    got = _decode(q, kv)
    assert_within_abs_or_ulp(got, oracle_every_sequence(q, kv), torch.bfloat16)


@pytest.mark.parametrize("hq,hkv", [(32, 1), (32, 8), (32, 32)], ids=["mqa", "gqa", "mha"])
def test_config4_every_sequence_matches_the_oracle(hq, hkv):
    """Config 4's ragged batch of 128 (lengths uniform in [1, 32768] with 16k - 1, 16k, 16k + 1):
    the load-balanced planner splits long sequences over many CTAs and packs short ones."""
    from kernel_lab.kv_cache import config4_lengths, random_paged_pool

    lens = config4_lengths(128)
    assert len(lens) == 128 and lens[:3] == [16383, 16384, 16385] and max(lens) <= 32768 and min(lens) >= 1
    q, kv = random_paged_pool(lens, hq, hkv, 128, 16, dtype=torch.bfloat16, device="cuda", seed=4)
    got = _decode(q, kv)
    assert_within_abs_or_ulp(got, oracle_every_sequence(q, kv), torch.bfloat16)
