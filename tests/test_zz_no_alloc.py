"""kl_paged_decode_noalloc: decode for callers that cannot allocate device memory.

Some hosts of this library own all GPU memory themselves (a serving engine that splits the
device between weights and its KV-cache pool at start-up) or must not call an allocator
inside their step loop. For them the library keeps a fixed per-GPU scratch array of its
own. These tests call that entry point through the C ABI and check that it gives the
same output as kl_paged_decode with caller-owned scratch, on consecutive calls (the
array keeps the previous call's contents, so each call must clear what it needs).

Kept in a file that pytest collects last, so that a failure here stops a -x run only
after every other test has run; it passes alone and after the others.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.conftest import NORTH_STAR_MAX_ABS

pytestmark = pytest.mark.gpu

CUDA_ERROR_MEMORY_ALLOCATION = 2


def noalloc(out, q, kv, num_splits=0):
    from kernel_lab import capi

    lib = capi.load()
    b, hq, d = q.shape
    num_pages, page, hkv, _ = kv.k_cache.shape
    return lib.kl_paged_decode_noalloc(
        capi.DTYPE_CODES[q.dtype], out.data_ptr(), q.data_ptr(), kv.k_cache.data_ptr(), kv.v_cache.data_ptr(),
        kv.block_table.data_ptr(), kv.seq_lens.data_ptr(), b, hq, hkv, d, page, kv.block_table.stride(0),
        kv.block_table.shape[1], num_pages, d**-0.5, num_splits, torch.cuda.current_stream().cuda_stream,
    )


def with_scratch(q, kv, num_splits=0):
    from kernel_lab import capi

    out = torch.empty_like(q)
    capi.paged_decode(out, q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, num_splits=num_splits)
    return out


@pytest.mark.parametrize(
    "lens,hq,hkv,dtype,num_splits",
    [
        ([4096] * 8, 32, 8, torch.bfloat16, 0),  # Llama-3-8B heads, tensor-core path
        ([1, 15, 16, 17, 255, 1000], 32, 1, torch.bfloat16, 0),  # MQA, ragged
        ([5, 40, 3, 77], 8, 2, torch.float32, 3),  # generic CUDA-core path, forced splits
    ],
)
def test_noalloc_matches_caller_scratch_on_consecutive_calls(lens, hq, hkv, dtype, num_splits):
    from kernel_lab.kv_cache import random_paged_pool

    q, kv = random_paged_pool(lens, hq, hkv, 128, 16, dtype=dtype, device="cuda", seed=11)
    want = with_scratch(q, kv, num_splits)
    tol = NORTH_STAR_MAX_ABS[dtype]
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        assert noalloc(got, q, kv, num_splits) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got.float() - want.float()).abs().max().item() <= tol


def test_noalloc_consecutive_calls_of_different_shapes():
    """A smaller problem after a larger one: stale counters of the first must not leak."""
    from kernel_lab.kv_cache import random_paged_pool

    for lens in ([3000] * 16, [700, 20, 1], [3000] * 16):
        q, kv = random_paged_pool(lens, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=len(lens))
        got = torch.empty_like(q)
        assert noalloc(got, q, kv) == 0
        torch.cuda.synchronize()
        assert (got.float() - with_scratch(q, kv).float()).abs().max().item() <= NORTH_STAR_MAX_ABS[torch.bfloat16]


def test_noalloc_matches_the_oracle():
    """The no-allocation path against the fp32 oracle itself, not only against the other entry
    point: ragged lengths around page boundaries, Llama-3-8B heads, two calls in a row."""
    from oracle import oracle
    from kernel_lab.kv_cache import random_paged_pool
    from tests.conftest import assert_within_abs_or_ulp, to_f32_numpy

    lens = [1, 15, 16, 17, 300, 1025, 2048, 4095]
    q, kv = random_paged_pool(lens, 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=12)
    table = kv.block_table.cpu().numpy()
    want = oracle.paged_decode_attention(
        to_f32_numpy(q), to_f32_numpy(kv.k_cache), to_f32_numpy(kv.v_cache), table, kv.seq_lens.cpu().numpy(),
        None, "f32",
    )
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        assert noalloc(got, q, kv) == 0
        torch.cuda.synchronize()
        assert_within_abs_or_ulp(got, want, torch.bfloat16)


def test_noalloc_status_reader_reports_a_bad_page():
    """Status bits of a no-allocation call are read from the library's own array: a block-table
    entry past the pool is skipped and flagged KL_STATUS_BAD_PAGE, and the next call clears it."""
    import ctypes as C

    from kernel_lab import capi
    from kernel_lab.kv_cache import random_paged_pool

    lib = capi.load()
    stream = torch.cuda.current_stream().cuda_stream
    q, kv = random_paged_pool([100, 40], 32, 8, 128, 16, dtype=torch.bfloat16, device="cuda", seed=13)
    bad = kv.block_table.clone()
    bad[1, 1] = kv.k_cache.shape[0] + 5  # outside the pool: never followed
    bad_kv = type(kv)(kv.k_cache, kv.v_cache, bad, kv.seq_lens, 16)
    out = torch.empty_like(q)
    status = C.c_uint32(0xFFFF)
    assert noalloc(out, q, bad_kv) == 0
    assert lib.kl_paged_decode_noalloc_read_status(C.byref(status), 0, stream) == 0
    assert status.value == capi.KL_STATUS_BAD_PAGE
    assert noalloc(out, q, kv) == 0  # a clean call starts from a cleared word
    assert lib.kl_paged_decode_noalloc_read_status(C.byref(status), 1, stream) == 0
    assert status.value == 0
    # Sequence 0 never touches the bad entry: its output is still right.
    assert torch.equal(out[0], with_scratch(q, kv)[0])


def test_noalloc_rejects_problems_beyond_its_scratch():
    from kernel_lab import capi

    lib = capi.load()
    pb, sb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    # 4096 sequences x 64 forced splits x 8 KV heads of partials: far beyond 16 MiB.
    assert lib.kl_paged_decode_workspace_size(2, 4096, 32, 8, 128, 16, 256, 64, ctypes.byref(pb), ctypes.byref(sb)) == 0
    assert pb.value > 16 << 20
    q = torch.zeros(4096, 32, 128, device="cuda", dtype=torch.bfloat16)
    rc = lib.kl_paged_decode_noalloc(2, q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                     q.data_ptr(), 4096, 32, 8, 128, 16, 256, 256, 1, 0.1, 64,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == CUDA_ERROR_MEMORY_ALLOCATION
