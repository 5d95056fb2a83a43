"""Failure detection of the fused head gather, on one GPU, without a fault.

A rank of a two-rank gather whose peer never arrives: the peer's output region and flags are
local buffers that nothing else writes, so the kernel's bounded wait for the peer's arrival runs
out (``timeout_ms``, read on the GPU's global timer). The kernel then sets KL_STATUS_PEER_TIMEOUT,
which the host reads, and returns; the context stays usable, and the next call, whose peer flag
the host has set, completes with status 0. One kernel, one GPU: nothing else waits on it.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_missing_peer_times_out_with_a_status_and_the_next_call_succeeds():
    from kernel_lab import capi, cuda_ops
    from kernel_lab.kv_cache import random_paged_pool

    q, kv = random_paged_pool([700, 33, 4096, 1, 16], 8, 2, 128, 16, dtype=torch.bfloat16, device="cuda", seed=21)
    scale = 128**-0.5
    # Rank 0 of 2 holds query heads [0, 4) and KV head 0.
    q0 = q[:, :4].contiguous()
    k0, v0 = kv.k_cache[:, :, :1].contiguous(), kv.v_cache[:, :, :1].contiguous()
    want = cuda_ops.paged_decode_attention(q0, k0, v0, kv.block_table, kv.seq_lens, scale)

    out_own = torch.full_like(q, float("nan"))
    out_peer = torch.full_like(q, float("nan"))  # stands in for rank 1's output as mapped here
    flags = torch.zeros(2, 2, dtype=torch.int32, device="cuda")  # flags[r]: rank r's arrivals
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = capi.HeadGather()
    g.num_ranks, g.rank, g.epoch, g.timeout_ms = 2, 0, 1, 200
    g.out[0], g.out[1] = out_own.data_ptr(), out_peer.data_ptr()
    g.flags[0], g.flags[1] = flags[0].data_ptr(), flags[1].data_ptr()
    g.done = done.data_ptr()
    scratch = capi.DecodeScratch.for_problem(q0, k0, kv.block_table)

    torch.cuda.synchronize()
    t0 = time.monotonic()
    capi.paged_decode_gather(g, q0, k0, v0, kv.block_table, kv.seq_lens, scale, scratch)
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert scratch.status(clear=True) == capi.KL_STATUS_PEER_TIMEOUT
    assert 0.15 < elapsed < 5.0, elapsed
    # This rank's heads are stored in both outputs; the absent peer's heads are not.
    assert torch.equal(out_own[:, :4], want) and torch.equal(out_peer[:, :4], want)
    assert out_own[:, 4:].isnan().all()
    # It published its arrival in both ranks' flags and returned its CTA count to zero.
    assert flags[:, 0].tolist() == [1, 1] and flags[0, 1].item() == 0 and done.item() == 0

    # The peer arrives for the next call (epoch 2): no timeout, and the output is the same.
    flags[0, 1] = 2
    g.epoch = 2
    out_own.fill_(float("nan"))
    t0 = time.monotonic()
    capi.paged_decode_gather(g, q0, k0, v0, kv.block_table, kv.seq_lens, scale, scratch)
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 0.15
    assert scratch.status(clear=True) == 0
    assert torch.equal(out_own[:, :4], want)
    assert flags[:, 0].tolist() == [2, 2] and done.item() == 0
