"""Cascade (shared-prefix) decode on the GPU against the oracle.

Groups of consecutive sequences share a prefix held in its own pages; each sequence attends to
its group's prefix and then to its own tokens. The kernel reads a prefix once per block of its
group's sequences and merges the two parts by their log-sum-exp in the same launch; the oracle
attends over the concatenated token list (oracle.paged_decode_attention_cascade, itself pinned to
the decode oracle). Bound: the north star's max-abs 2e-3 (fp16) / 2e-2 (bf16), or one storage
ulp where the output is large. Spare pages are NaN and never read.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import assert_within_abs_or_ulp

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["tensor_core_prefix", "prefix_in_plan"])
def prefix_path(request, monkeypatch):
    """Both ways a prefix is computed, forced: the tcgen05 prefix kernel (KL_DECODE_CASCADE_TC=1,
    where its shapes fit) and prefix items inside the decode kernel's plan (=0)."""
    monkeypatch.setenv("KL_DECODE_CASCADE_TC", "0" if request.param == "prefix_in_plan" else "1")
    return request.param

KL_STATUS_BAD_PAGE = 1
KL_STATUS_BAD_PREFIX_GROUPS = 8


def _problem(group_sizes, prefix_lens, seq_lens, hq, hkv, d, page, dtype, seed=0):
    from kernel_lab.kv_cache import random_cascade_problem

    return random_cascade_problem(group_sizes, prefix_lens, seq_lens, hq, hkv, d, page, dtype=dtype, device="cuda",
                                  seed=seed)


def _oracle(q, kv, k_cache=None, v_cache=None):
    k = (kv.k_cache if k_cache is None else k_cache).float().cpu().numpy()
    v = (kv.v_cache if v_cache is None else v_cache).float().cpu().numpy()
    return oracle.paged_decode_attention_cascade(
        q.float().cpu().numpy(), k, v, kv.prefix_block_table.cpu().numpy(), kv.prefix_lens.cpu().numpy(),
        kv.prefix_indptr.cpu().numpy(), kv.block_table.cpu().numpy(), kv.seq_lens.cpu().numpy(),
    )


def _run(q, kv, **kw):
    from kernel_lab import cuda_ops

    return cuda_ops.paged_decode_attention_cascade(
        q, kv.k_cache if "k_cache" not in kw else kw.pop("k_cache"),
        kv.v_cache if "v_cache" not in kw else kw.pop("v_cache"), kv.prefix_block_table, kv.prefix_lens,
        kv.prefix_indptr, kv.block_table, kv.seq_lens, **kw,
    )


CASES = [
    # (group sizes, prefix lens, own lens, hq, hkv, d, page)
    ([4], [64], [1, 17, 33, 70], 32, 8, 128, 16),
    # ragged prefixes, an empty group, a group without a prefix, sequences without own tokens
    ([3, 1, 0, 4], [37, 0, 24, 300], [5, 0, 9, 17, 1, 8, 0, 30], 32, 8, 128, 16),
    # MHA (group 1): eight sequences' rows share each prefix MMA
    ([5, 3], [1000, 129], [3, 200, 17, 1, 64, 500, 2, 33], 32, 32, 128, 16),
    ([6], [250], [7, 64, 200, 1, 0, 13], 16, 4, 64, 8),
    ([2, 2], [513, 40], [9, 250, 0, 31], 32, 8, 256, 16),
    # MQA (group 32): one sequence per prefix item, two query-head groups per KV head
    ([3], [2000], [17, 1, 450], 32, 1, 128, 32),
    ([9], [128], [5, 9, 33, 1, 64, 7, 100, 2, 16], 64, 8, 128, 16),
    # long prefix, tiny batch: the prefix item is split over many CTAs (flat merge into the cascade)
    ([2], [8192], [100, 3000], 32, 8, 128, 16),
    # everything empty but one sequence
    ([1, 2], [0, 0], [0, 0, 5], 32, 8, 128, 16),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cascade_matches_the_oracle(case, dtype, prefix_path):
    from kernel_lab import cuda_ops

    groups, plens, lens, hq, hkv, d, page = CASES[case]
    q, kv = _problem(groups, plens, lens, hq, hkv, d, page, dtype, seed=case)
    cuda_ops.decode_status(clear=True)
    got = _run(q, kv)
    torch.cuda.synchronize()
    assert cuda_ops.decode_status(clear=True) == 0
    assert_within_abs_or_ulp(got, _oracle(q, kv), dtype)


def test_cascade_is_deterministic_and_leaves_scratch_reusable(prefix_path):
    """Same inputs, same bits, whichever side of a cascade finishes second; a second call on
    the same scratch (counters returned to zero) gives the same result."""
    from kernel_lab import capi

    q, kv = _problem([2, 5], [4096, 777], [100, 3000, 1, 17, 250, 0, 64], 32, 8, 128, 16, torch.bfloat16, seed=11)
    out1, out2 = torch.empty_like(q), torch.empty_like(q)
    args = (kv.k_cache, kv.v_cache, kv.prefix_block_table, kv.prefix_lens, kv.prefix_indptr, kv.block_table,
            kv.seq_lens)
    scratch = capi.paged_decode_cascade(out1, q, *args)
    for _ in range(3):
        capi.paged_decode_cascade(out2, q, *args, scratch=scratch)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2)
    assert scratch.status(clear=True) == 0


def test_cascade_equals_plain_decode_over_concatenated_tables_at_serving_size(prefix_path):
    """Headline shapes: 64 sequences share a 4096-token prefix and own 512 tokens each. The same
    problem without sharing (each row lists the prefix pages, then its own) through the plain
    decode op agrees within the two kernels' combined rounding."""
    from kernel_lab import cuda_ops

    q, kv = _problem([64], [4096], [512] * 64, 32, 8, 128, 16, torch.bfloat16, seed=2)
    got = _run(q, kv)
    table, lens = kv.concatenated_tables()
    ref = cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, table, lens)
    assert torch.isfinite(got).all()
    assert (got.float() - ref.float()).abs().max().item() <= 2e-2


def test_cascade_with_bad_groups_ignores_prefixes_and_says_so(prefix_path):
    from kernel_lab import cuda_ops

    q, kv = _problem([2, 2], [64, 32], [10, 20, 30, 40], 32, 8, 128, 16, torch.bfloat16, seed=4)
    kv.prefix_indptr = torch.tensor([0, 3, 3], dtype=torch.int32, device="cuda")  # ends before the batch does
    cuda_ops.decode_status(clear=True)
    got = _run(q, kv)
    torch.cuda.synchronize()
    assert cuda_ops.decode_status(clear=True) & KL_STATUS_BAD_PREFIX_GROUPS
    assert_within_abs_or_ulp(got, _oracle(q, kv), torch.bfloat16)


def test_cascade_bad_prefix_page_is_skipped_and_flagged(prefix_path):
    from kernel_lab import cuda_ops

    q, kv = _problem([3], [64], [10, 20, 30], 32, 8, 128, 16, torch.bfloat16, seed=6)
    kv.prefix_block_table[0, 1] = kv.k_cache.shape[0] + 5  # outside the pool
    cuda_ops.decode_status(clear=True)
    got = _run(q, kv)
    torch.cuda.synchronize()
    assert cuda_ops.decode_status(clear=True) & KL_STATUS_BAD_PAGE
    assert torch.isfinite(got).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cascade_over_an_e4m3_cache(dtype):
    from kernel_lab.kv_cache import e4m3_scales, quantize_e4m3

    q, kv = _problem([3, 4], [300, 1000], [5, 64, 0, 17, 200, 1, 33], 32, 8, 128, 16, dtype, seed=8)
    ks, vs = e4m3_scales(kv.k_cache), e4m3_scales(kv.v_cache)
    k8, v8 = quantize_e4m3(kv.k_cache, ks), quantize_e4m3(kv.v_cache, vs)
    got = _run(q, kv, k_cache=k8, v_cache=v8, k_scale=ks, v_scale=vs)
    kd = k8.float() * ks.view(1, 1, -1, 1)
    vd = v8.float() * vs.view(1, 1, -1, 1)
    assert_within_abs_or_ulp(got, _oracle(q, kv, kd, vd), dtype)
