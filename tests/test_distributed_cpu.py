"""KV-head-sharded decode across ranks, on CPU with the gloo backend (world size 2).

The sharded step is: local attention over this rank's KV heads, then one all-gather of the
per-rank outputs re-laid into [B, Hq, D]. Here the local attention is the oracle (these ranks
have no GPU); what is under test is the host logic: head ranges, shard slicing, gather and
re-layout must reproduce the unsharded result exactly. A second test makes one rank fail on
the host before the collective and checks that the other rank gets an error from the short
process-group timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (REPO, os.path.join(REPO, "kernel-lab_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _oracle_decode(q, k, v, bt, lens, scale):
    from oracle import oracle

    out = oracle.paged_decode_attention(q.numpy(), k.numpy(), v.numpy(), bt.numpy(), lens.numpy(), scale, "f32")
    return torch.from_numpy(out)


def _sharded_worker(rank, world, port, result_q):
    _paths()
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from kernel_lab.kv_cache import random_decode_problem
        from kernel_lab.sharding import ShardedPagedDecode, shard_heads

        q, kv, _, _ = random_decode_problem([7, 33, 100], 16, 4, 32, 16, dtype=torch.float32, seed=3)
        q_l, k_l, v_l = shard_heads(q, kv.k_cache, kv.v_cache, world, rank)
        step = ShardedPagedDecode(local_decode=_oracle_decode)
        full = step(q_l, k_l, v_l, kv.block_table, kv.seq_lens, 32**-0.5)
        want = _oracle_decode(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, 32**-0.5)
        result_q.put((rank, float((full - want).abs().max()), tuple(full.shape)))
        dist.destroy_process_group()
    except Exception:
        result_q.put((rank, traceback.format_exc(), None))


def test_sharded_decode_matches_unsharded_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err, shape in results:
        assert shape == (3, 16, 32), f"rank {rank}: {err}"
        assert err == 0.0


def _failing_worker(rank, world, port, result_q):
    _paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from kernel_lab.sharding import gather_heads

    if rank == 1:
        # A host-side failure before this rank's collective: it leaves without gathering.
        result_q.put((rank, "left"))
        return
    try:
        gather_heads(torch.zeros(2, 4, 8), world)
        result_q.put((rank, "no error"))
    except Exception as exc:  # the gloo timeout (or the peer's disconnect) surfaces here
        result_q.put((rank, f"error: {type(exc).__name__}"))


def test_a_rank_that_leaves_makes_the_collective_fail_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error"), results[0]


def test_head_ranges_and_shards_cover_the_problem():
    _paths()
    from kernel_lab.kv_cache import random_decode_problem
    from kernel_lab.sharding import gather_heads, kv_head_range, shard_heads

    assert [kv_head_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    from kernel_lab.sharding import batch_range

    assert [batch_range(10, 4, r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert [batch_range(128, 2, r) for r in range(2)] == [(0, 64), (64, 128)]
    try:
        kv_head_range(8, 3, 0)
        raise AssertionError("uneven sharding must be rejected")
    except ValueError:
        pass
    q, kv, _, _ = random_decode_problem([9, 20], 32, 8, 16, 16, dtype=torch.float32)
    parts = [shard_heads(q, kv.k_cache, kv.v_cache, 4, r) for r in range(4)]
    np.testing.assert_array_equal(torch.cat([p[0] for p in parts], dim=1).numpy(), q.numpy())
    np.testing.assert_array_equal(torch.cat([p[1] for p in parts], dim=2).numpy(), kv.k_cache.numpy())
    # world size 1: the gather is the identity.
    assert gather_heads(q, 1) is q


def _exchange_worker(rank, world, port, result_q):
    _paths()
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from kernel_lab.sharding import exchange, require_distinct_devices

        # Handles of the fused head gather's buffers (64 bytes each) reach every rank in rank order.
        handles = exchange(bytes([rank]) * 64)
        # Two ranks that report one GPU are refused before any kernel could wait on the other.
        refused = False
        try:
            require_distinct_devices(exchange("same-gpu"))
        except RuntimeError:
            refused = True
        require_distinct_devices(exchange(f"gpu-{rank}"))
        dist.destroy_process_group()
        result_q.put((rank, handles == [bytes([r]) * 64 for r in range(world)], refused, None))
    except Exception:
        result_q.put((rank, False, False, traceback.format_exc()))


def test_fused_gather_host_logic_on_gloo_ranks():
    """The host side of PeerHeadGather across two CPU ranks: IPC handles exchanged in rank order,
    ranks on one device refused, and the call numbers (epochs) that key the output regions."""
    _paths()
    from kernel_lab.sharding import next_epoch

    assert next_epoch(0) == 1 and next_epoch(7) == 8
    assert next_epoch((1 << 32) - 1) == 1  # 0 is never a call number
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ordered, refused, err in results:
        assert err is None, f"rank {rank}: {err}"
        assert ordered and refused
