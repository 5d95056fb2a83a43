"""Multi-GPU layouts of decode attention (one process per GPU, NCCL over NVLink).

By sequence (``batch_range``): sequences are independent, so each rank decodes its own and
nothing is exchanged. By KV head (tensor parallel, below):

A KV head and the query heads of its group need no data from any other head, so the
heads shard with no exchange during the attention itself: rank r of N keeps KV heads
[r*Hkv/N, (r+1)*Hkv/N) of the paged pool (its own contiguous pool; the block table and
seq_lens are replicated) and query heads [r*Hq/N, (r+1)*Hq/N). The one exchange is the
gather of every rank's heads into the full [B, Hq, D] output on every rank:

* ``PeerHeadGather`` (the product path): the decode kernel itself stores each final row into
  every rank's output over NVLink (plain peer stores into CUDA-IPC-mapped buffers, no multicast)
  and ends with one cross-GPU arrival, so one launch per step does the attention and the gather.
* ``gather_heads`` / ``ShardedPagedDecode``: the library baseline, the single-GPU op followed by
  one NCCL all-gather into [N, B, Hq/N, D] and a permuting copy to [B, Hq, D].

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


def _align(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def exchange(obj, group=None) -> list:
    """Every rank's `obj`, in rank order (one all-gather of Python objects over the group)."""
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def require_distinct_devices(device_ids: list[str]) -> None:
    """The ranks of a head gather wait on one another inside the kernel, so no two may share a GPU."""
    if len(set(device_ids)) != len(device_ids):
        raise RuntimeError(f"the ranks of a head gather must run on distinct GPUs, got {device_ids}")


def next_epoch(epoch: int) -> int:
    """The call number after `epoch`: 1, 2, ... 2**32 - 1, then 1 again (0 is never used)."""
    return 1 if epoch >= (1 << 32) - 1 else epoch + 1


class PeerHeadGather:
    """One rank's KV-head-sharded decode with the head gather fused into the kernel.

    Each rank owns one buffer (``kl_ipc_alloc``) holding ``slots`` output regions of the full
    [batch, N * num_q_heads, head_dim] and the gather's flags; the other ranks map it
    (``kl_ipc_open``, handles exchanged once over the process group). A call passes this rank's
    query heads and KV-head pool; ``kl_paged_decode_gather`` stores every final row into the
    current region of every rank's buffer and returns once all ranks' rows have arrived, so the
    returned tensor (a view of this rank's region) is the whole output. Regions rotate by call
    number: the output of a call stays valid until the call two after it runs on this rank's
    stream (a peer may be one call ahead). Every rank must make the same calls in the same
    order, on distinct GPUs. With one rank it is the plain decode into a local region.
    A rank whose peers do not arrive within ``timeout_ms`` (0: 10 s) returns with
    ``KL_STATUS_PEER_TIMEOUT`` in ``status()``.
    """

    def __init__(self, batch: int, num_q_heads: int, head_dim: int, dtype: torch.dtype = torch.bfloat16,
                 group=None, slots: int = 3, timeout_ms: int = 0):
        from kernel_lab import capi

        if slots < 2:
            raise ValueError("a head gather needs at least two output regions")
        self.capi = capi
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > capi.KL_GATHER_MAX_RANKS:
            raise ValueError(f"a head gather spans at most {capi.KL_GATHER_MAX_RANKS} ranks")
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.shape = (batch, self.world * num_q_heads, head_dim)
        self.dtype = dtype
        self.slots = slots
        elem = torch.empty((), dtype=dtype).element_size()
        self.region = _align(batch * self.world * num_q_heads * head_dim * elem, 256)
        flags_off = slots * self.region
        done_off = flags_off + 64
        total = done_off + 64
        self._local = None
        if self.world == 1:
            self._local = torch.zeros(total, dtype=torch.uint8, device=self.device)
            bases = [self._local.data_ptr()]
        else:
            # Ranks wait on one another inside the kernel: never two ranks on one GPU.
            require_distinct_devices(exchange(str(torch.cuda.get_device_properties(self.device).uuid), group))
            base, handle = capi.ipc_alloc(total)
            handles = exchange(handle, group)
            bases = [base if r == self.rank else capi.ipc_open(handles[r]) for r in range(self.world)]
            dist.barrier(group=group)
        self.bases = bases
        self.views = [capi.device_tensor(bases[self.rank] + k * self.region, self.shape, dtype, self.device)
                      for k in range(slots)]
        g = capi.HeadGather()
        g.num_ranks = self.world
        g.rank = self.rank
        for r in range(self.world):
            g.flags[r] = bases[r] + flags_off
        g.done = bases[self.rank] + done_off
        g.timeout_ms = timeout_ms
        self._g = g
        self.epoch = 0
        self.scratch = None
        self._scratch_key = None

    def __call__(self, q_local, k_local, v_local, block_table, seq_lens, scale=None) -> torch.Tensor:
        """This rank's shard of the step; returns the full [batch, Hq, head_dim] output (a view)."""
        if tuple(q_local.shape) != (self.shape[0], self.shape[1] // self.world, self.shape[2]) or \
                q_local.dtype != self.dtype:
            raise ValueError(f"q is {tuple(q_local.shape)} {q_local.dtype}; this gather was set up for "
                             f"{(self.shape[0], self.shape[1] // self.world, self.shape[2])} {self.dtype}")
        key = (tuple(k_local.shape), block_table.shape[1])
        if self._scratch_key != key:
            self.scratch = self.capi.DecodeScratch.for_problem(q_local, k_local, block_table)
            self._scratch_key = key
        self.epoch = next_epoch(self.epoch)
        slot = self.epoch % self.slots
        g = self._g
        g.epoch = self.epoch
        for r in range(self.world):
            g.out[r] = self.bases[r] + slot * self.region
        self.capi.paged_decode_gather(g, q_local, k_local, v_local, block_table, seq_lens, scale, self.scratch)
        return self.views[slot]

    def status(self, clear: bool = False) -> int:
        """KL_STATUS_* bits of this rank's calls (synchronises the current stream)."""
        return 0 if self.scratch is None else self.scratch.status(clear)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's, after every rank has finished its calls."""
        if self.bases is None:
            return
        torch.cuda.synchronize(self.device)
        self.views = []
        if self.world > 1:
            dist.barrier(group=self.group)
            for r, b in enumerate(self.bases):
                if r != self.rank:
                    self.capi.ipc_close(b)
            dist.barrier(group=self.group)
            self.capi.ipc_free(self.bases[self.rank])
        self.bases = None
        self._local = None
