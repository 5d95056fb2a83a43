"""KV-head-sharded decode on real GPUs: one process per GPU (config 5's layout).

Two gathers of the heads are tested: the product path, where the decode kernel stores its rows
into every rank's output over NVLink (``PeerHeadGather``), and the NCCL all-gather baseline.

Needs at least two visible GPUs; skipped otherwise. Each rank runs the single-GPU CUDA op on its
own KV heads; each rank's slice of the gathered output must equal its own local output bit for
bit (the gather and re-layout are exact), and the whole must match the unsharded op run on one
GPU within the bf16 tolerance (a rank plans its 4 KV heads into other chunks than the 8-head
plan, so the split-KV merges differ in rounding). The host logic of the same path, and its failure path (a rank that leaves makes the
collective fail on the short process-group timeout instead of hanging), are tested on CPU with
gloo ranks in test_distributed_cpu.py.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (REPO, os.path.join(REPO, "kernel-lab_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _problem(device, hq=64, hkv=8):
    from kernel_lab.kv_cache import random_paged_pool

    # Config 5's heads (64 query / 8 KV, D 128, bf16) on ragged lengths across page boundaries.
    lens = [1, 15, 16, 17, 300, 1025, 4096, 777]
    return random_paged_pool(lens, hq, hkv, 128, 16, dtype=torch.bfloat16, device=device, seed=21)


def _worker(rank, world, port, result_q):
    _paths()
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as dist

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from kernel_lab import cuda_ops
        from kernel_lab.sharding import ShardedPagedDecode, shard_heads

        q, kv = _problem(dev)
        q_l, k_l, v_l = shard_heads(q, kv.k_cache, kv.v_cache, world, rank)
        step = ShardedPagedDecode()
        got = step(q_l, k_l, v_l, kv.block_table, kv.seq_lens, 128**-0.5)
        local = cuda_ops.paged_decode_attention(q_l, k_l, v_l, kv.block_table, kv.seq_lens, 128**-0.5)
        want = cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, 128**-0.5)
        torch.cuda.synchronize()
        hq_l = q_l.shape[1]
        same = bool(torch.equal(got[:, rank * hq_l : (rank + 1) * hq_l], local))
        close = bool(torch.allclose(got.float(), want.float(), atol=1.6e-2, rtol=1.6e-2))
        status = cuda_ops.decode_status(clear=True)
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, same and close, status, None if same and close else f"slice exact {same}, close {close}"))
    except Exception:
        result_q.put((rank, False, -1, traceback.format_exc()))


def test_sharded_decode_on_two_gpus_matches_the_unsharded_op():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, same, status, err in results:
        assert err is None, f"rank {rank}: {err}"
        assert same, f"rank {rank}: sharded output differs from the unsharded op"
        assert status == 0


def _peer_worker(rank, world, port, result_q, hq=64, hkv=8):
    _paths()
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as dist

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from kernel_lab import cuda_ops
        from kernel_lab.sharding import PeerHeadGather, gather_heads, shard_heads

        errors = []
        q, kv = _problem(dev, hq, hkv)
        q_l, k_l, v_l = shard_heads(q, kv.k_cache, kv.v_cache, world, rank)
        want = cuda_ops.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, 128**-0.5)
        local = cuda_ops.paged_decode_attention(q_l, k_l, v_l, kv.block_table, kv.seq_lens, 128**-0.5)
        nccl = gather_heads(local, world)
        gather = PeerHeadGather(q.shape[0], q_l.shape[1], 128, torch.bfloat16)
        hq_l = q_l.shape[1]
        # Five calls in a row (regions rotate), each checked before the next one is enqueued; the
        # third call gets a different q (scaled), so stale rows from an earlier call would show.
        for call in range(5):
            qc = q_l * 0.5 if call == 2 else q_l
            got = gather(qc, k_l, v_l, kv.block_table, kv.seq_lens, 128**-0.5)
            torch.cuda.synchronize()
            if call == 2:
                ref_local = cuda_ops.paged_decode_attention(qc, k_l, v_l, kv.block_table, kv.seq_lens, 128**-0.5)
                if not torch.equal(got[:, rank * hq_l : (rank + 1) * hq_l], ref_local):
                    errors.append(f"call {call}: own heads differ from the local op")
                continue
            if not torch.equal(got[:, rank * hq_l : (rank + 1) * hq_l], local):
                errors.append(f"call {call}: own heads differ from the local op")
            if not torch.equal(got, nccl):
                errors.append(f"call {call}: differs from the NCCL all-gather of the same shards")
            if not torch.allclose(got.float(), want.float(), atol=1.6e-2, rtol=1.6e-2):
                errors.append(f"call {call}: not close to the unsharded op")
        status = gather.status(clear=True)
        gather.close()
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, not errors, status, "; ".join(errors) or None))
    except Exception:
        result_q.put((rank, False, -1, traceback.format_exc()))


@pytest.mark.parametrize("hq,hkv", [(64, 8), (8, 2)], ids=["4_kv_heads_a_rank", "1_kv_head_a_rank"])
def test_fused_peer_gather_on_two_gpus_matches_nccl_and_the_unsharded_op(hq, hkv):
    """With one KV head a rank (as Llama-3 heads sharded 8 ways) each warp of the kernel walks its
    own stream of the plan; with four, the warps of a tile share one ring."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q, hq, hkv)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, status, err in results:
        assert err is None, f"rank {rank}: {err}"
        assert ok
        assert status == 0
