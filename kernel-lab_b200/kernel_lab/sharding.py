"""Multi-GPU layouts of decode attention (one process per GPU, NCCL over NVLink).

By sequence (``batch_range``): sequences are independent, so each rank decodes its own and
nothing is exchanged. By KV head (tensor parallel, below):

A KV head and the query heads of its group need no data from any other head, so the
heads shard with no exchange during the attention itself: rank r of N keeps KV heads
[r*Hkv/N, (r+1)*Hkv/N) of the paged pool (its own contiguous pool; the block table and
seq_lens are replicated) and query heads [r*Hq/N, (r+1)*Hq/N), and runs the single-GPU
kernel unchanged. The one collective is an all-gather of the per-rank outputs
[B, Hq/N, D] into [N, B, Hq/N, D], re-laid to [B, Hq, D].

kernel-lab itself is single-GPU; this is the multi-GPU layout of its decode op.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist


def kv_head_range(num_kv_heads: int, world_size: int, rank: int) -> tuple[int, int]:
    """KV heads [lo, hi) owned by `rank`; the heads must divide evenly."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} of {world_size}")
    if num_kv_heads % world_size:
        raise ValueError(f"{num_kv_heads} KV heads do not shard evenly over {world_size} ranks")
    per = num_kv_heads // world_size
    return rank * per, (rank + 1) * per


def batch_range(batch: int, world_size: int, rank: int) -> tuple[int, int]:
    """Sequences [lo, hi) decoded by `rank` when the batch is split instead of the heads
    (sequences are independent: no collective). Uneven batches give the first ranks one more."""
    if world_size <= 0 or not 0 <= rank < world_size or batch < 0:
        raise ValueError(f"bad rank {rank} of {world_size} for batch {batch}")
    per, extra = divmod(batch, world_size)
    lo = rank * per + min(rank, extra)
    return lo, lo + per + (1 if rank < extra else 0)


def shard_heads(
    q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, world_size: int, rank: int
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Slice one rank's query heads [B, Hq/N, D] and KV pool [P, page, Hkv/N, D] (contiguous copies)."""
    num_kv_heads = k_cache.shape[2]
    group = q.shape[1] // num_kv_heads
    lo, hi = kv_head_range(num_kv_heads, world_size, rank)
    return (
        q[:, lo * group : hi * group].contiguous(),
        k_cache[:, :, lo:hi].contiguous(),
        v_cache[:, :, lo:hi].contiguous(),
    )


_GATHER_BUFFERS: dict[tuple, torch.Tensor] = {}


def gather_heads(local_out: torch.Tensor, world_size: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather per-rank outputs [B, Hq/N, D] and return the full [B, Hq, D] in head order.

    The collective lands in a cached [N, B, Hq/N, D] buffer (one per shape, device and group);
    one permuting copy then writes `out` (allocated if not given)."""
    if world_size == 1:
        if out is not None:
            out.copy_(local_out)
            return out
        return local_out
    b, hl, d = local_out.shape
    key = (world_size, b, hl, d, local_out.dtype, local_out.device, id(group))
    stacked = _GATHER_BUFFERS.get(key)
    if stacked is None:
        stacked = torch.empty((world_size * b, hl, d), dtype=local_out.dtype, device=local_out.device)
        _GATHER_BUFFERS[key] = stacked
    dist.all_gather_into_tensor(stacked, local_out.contiguous(), group=group)
    if out is None:
        out = torch.empty((b, world_size * hl, d), dtype=local_out.dtype, device=local_out.device)
    out.view(b, world_size, hl, d).copy_(stacked.view(world_size, b, hl, d).permute(1, 0, 2, 3))
    return out


class ShardedPagedDecode:
    """One rank's step of KV-head-sharded decode: local attention, then the all-gather.

    ``local_decode(q, k_cache, v_cache, block_table, seq_lens, scale) -> out`` defaults to
    the CUDA op; tests on CPU ranks pass the oracle instead.
    """

    def __init__(self, group=None, local_decode: Callable | None = None):
        self.group = group
        self.world_size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if local_decode is None:
            from kernel_lab import cuda_ops

            local_decode = cuda_ops.paged_decode_attention
        self.local_decode = local_decode

    def __call__(self, q_local, k_local, v_local, block_table, seq_lens, scale=None, out=None) -> torch.Tensor:
        local = self.local_decode(q_local, k_local, v_local, block_table, seq_lens, scale)
        return gather_heads(local, self.world_size, self.group, out)
