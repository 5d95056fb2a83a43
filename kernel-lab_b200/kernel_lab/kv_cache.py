"""Paged KV-cache pools: the data format on both sides of the decode kernel.

A serving engine keeps every sequence's keys and values in fixed-size pages of
one pool, NHD layout ``[num_pages, page_size, num_kv_heads, head_dim]``, and a
block table lists each sequence's pages in order. This module builds such pools.

``random_decode_problem`` / ``build_paged_kv`` reproduce the seeded fixtures of
kernel_lab/kv_cache.py:33-102 bit for bit (same generator protocol: one
``torch.Generator().manual_seed(seed)`` drawing q, then every sequence's keys,
then every sequence's values; a second one drawing the page permutation), so the
golden vectors produced by the reference apply to them. Two differences, both
deliberate: the spare-page poison is a parameter (default NaN, so a kernel that
reads a page it should not turns the output into NaN, not merely "large"), and
the scatter is vectorised instead of a per-page loop.

``random_paged_pool`` builds the large serving-scale pools for the benchmark
directly on the device (same layout and page shuffling, values from a CUDA
generator), because drawing gigabytes on the host would take minutes.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

NAN = float("nan")


@dataclass
class PagedKV:
    k_cache: torch.Tensor  # [num_pages, page_size, num_kv_heads, head_dim]
    v_cache: torch.Tensor
    block_table: torch.Tensor  # [batch, max_pages] int32, padded with page 0
    seq_lens: torch.Tensor  # [batch] int32
    page_size: int

    @property
    def max_pages(self) -> int:
        return self.block_table.shape[1]

    @property
    def num_pages(self) -> int:
        return self.k_cache.shape[0]


def config4_lengths(batch: int = 128, seed: int = 4) -> list[int]:
    """Config 4's ragged batch: lengths uniform in [1, 32768] from a seeded generator, the first
    three replaced by 16k - 1, 16k and 16k + 1 (at and around a multiple of the page size)."""
    import numpy as np

    rng = np.random.default_rng(seed)
    return [16383, 16384, 16385] + rng.integers(1, 32769, size=batch - 3).tolist()


def pages_for(seq_len: int, page_size: int) -> int:
    return (seq_len + page_size - 1) // page_size


def _page_order(total: int, seed: int) -> torch.Tensor:
    return torch.randperm(total, generator=torch.Generator().manual_seed(seed))


def build_paged_kv(
    keys: list[torch.Tensor],
    values: list[torch.Tensor],
    page_size: int,
    extra_pages: int = 3,
    seed: int = 0,
    poison: float = NAN,
) -> PagedKV:
    """Scatter per-sequence K/V (``[L, Hkv, D]`` each) into shuffled pages of one pool.

    Pages are handed out in the order of a seeded permutation of the pool; the
    ``extra_pages`` pages left over are filled with ``poison``; the unused tail of
    a sequence's last page is zero; block-table padding is page id 0.
    """
    if not keys or len(keys) != len(values):
        raise ValueError("need one K and one V tensor per sequence")
    _, num_kv_heads, head_dim = keys[0].shape
    lens = [k.shape[0] for k in keys]
    if min(lens) < 1:
        raise ValueError("every sequence needs at least one cached token")
    needed = [pages_for(n, page_size) for n in lens]
    used = sum(needed)
    total = used + extra_pages
    device, dtype = keys[0].device, keys[0].dtype

    order = _page_order(total, seed)
    table = torch.zeros((len(keys), max(needed)), dtype=torch.int32)
    starts = torch.tensor([0, *needed[:-1]]).cumsum(0)
    for b, n in enumerate(needed):
        table[b, :n] = order[starts[b] : starts[b] + n].to(torch.int32)

    # Destination (page, slot) of every token, all sequences concatenated.
    tok_page = torch.cat([table[b, torch.arange(n) // page_size].long() for b, n in enumerate(lens)])
    tok_slot = torch.cat([torch.arange(n) % page_size for n in lens])

    k_cache = torch.full((total, page_size, num_kv_heads, head_dim), poison, dtype=dtype, device=device)
    v_cache = torch.full_like(k_cache, poison)
    assigned = order[:used].to(device)
    k_cache[assigned] = 0  # partial-page tails: valid memory, never attended
    v_cache[assigned] = 0
    k_cache[tok_page.to(device), tok_slot.to(device)] = torch.cat(keys)
    v_cache[tok_page.to(device), tok_slot.to(device)] = torch.cat(values)
    return PagedKV(
        k_cache=k_cache,
        v_cache=v_cache,
        block_table=table.to(device),
        seq_lens=torch.tensor(lens, dtype=torch.int32, device=device),
        page_size=page_size,
    )


def random_decode_problem(
    seq_lens: list[int],
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    page_size: int,
    dtype: torch.dtype = torch.float16,
    device: str = "cpu",
    seed: int = 0,
    poison: float = NAN,
) -> tuple[torch.Tensor, PagedKV, list[torch.Tensor], list[torch.Tensor]]:
    """A seeded query batch and its paged cache, plus the contiguous K/V it came from.

    Values are N(0, 1) drawn in float32 on the host and rounded to ``dtype``.
    """
    generator = torch.Generator().manual_seed(seed)

    def rand(*shape: int) -> torch.Tensor:
        return torch.randn(*shape, generator=generator).to(device=device, dtype=dtype)

    q = rand(len(seq_lens), num_q_heads, head_dim)
    keys = [rand(n, num_kv_heads, head_dim) for n in seq_lens]
    values = [rand(n, num_kv_heads, head_dim) for n in seq_lens]
    return q, build_paged_kv(keys, values, page_size, seed=seed, poison=poison), keys, values


def random_paged_pool(
    seq_lens: list[int],
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    page_size: int,
    dtype: torch.dtype = torch.bfloat16,
    device: str | torch.device = "cuda",
    seed: int = 0,
    extra_pages: int = 3,
    poison: float = NAN,
    kv_head_slice: tuple[int, int] | None = None,
) -> tuple[torch.Tensor, PagedKV]:
    """Serving-scale pool generated on ``device``: N(0,1) q/K/V, shuffled pages, poisoned spares.

    ``kv_head_slice=(lo, hi)`` keeps only KV heads ``lo..hi-1`` (and their query
    groups) of the full problem, as one tensor-parallel rank holds them. Every
    rank draws the same full-size random stream per page, so the union of the
    shards is the unsharded problem.
    """
    dev = torch.device(device)
    lens = [int(n) for n in seq_lens]
    needed = [pages_for(n, page_size) for n in lens]
    used = sum(needed)
    total = used + extra_pages
    lo, hi = kv_head_slice if kv_head_slice is not None else (0, num_kv_heads)
    group = num_q_heads // num_kv_heads

    gen = torch.Generator(device=dev).manual_seed(seed)
    q_full = torch.randn(len(lens), num_q_heads, head_dim, generator=gen, device=dev, dtype=torch.float32)
    q = q_full[:, lo * group : hi * group].to(dtype).contiguous()

    shape = (total, page_size, hi - lo, head_dim)
    k_cache = torch.empty(shape, dtype=dtype, device=dev)
    v_cache = torch.empty(shape, dtype=dtype, device=dev)
    # Draw page-sized blocks of the full-width pool and keep this rank's heads, in
    # chunks so the float32 staging buffer stays small.
    chunk = max(1, (1 << 28) // (page_size * num_kv_heads * head_dim * 4))
    for start in range(0, total, chunk):
        stop = min(total, start + chunk)
        for cache in (k_cache, v_cache):
            block = torch.randn(
                stop - start, page_size, num_kv_heads, head_dim, generator=gen, device=dev, dtype=torch.float32
            )
            cache[start:stop] = block[:, :, lo:hi].to(dtype)
            del block

    order = _page_order(total, seed).to(dev)
    width = max(needed)
    table = torch.zeros((len(lens), width), dtype=torch.int32, device=dev)
    starts = torch.tensor([0, *needed[:-1]], device=dev).cumsum(0)
    cols = torch.arange(width, device=dev)
    need_t = torch.tensor(needed, device=dev)
    mask = cols[None, :] < need_t[:, None]
    src = (starts[:, None] + cols[None, :]).clamp(max=max(used - 1, 0))
    table = torch.where(mask, order[src].to(torch.int32), table)

    spare = order[used:]
    k_cache[spare] = poison
    v_cache[spare] = poison
    # Zero the unused tail of each sequence's last page.
    for b, n in enumerate(lens):
        tail = n % page_size
        if tail:
            page = int(order[int(starts[b]) + needed[b] - 1])
            k_cache[page, tail:] = 0
            v_cache[page, tail:] = 0
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    return q, PagedKV(k_cache=k_cache, v_cache=v_cache, block_table=table, seq_lens=seq, page_size=page_size)


@dataclass
class CascadeKV:
    """A paged pool holding shared prefixes and per-sequence tokens, with the cascade tables:
    group p = sequences prefix_indptr[p] .. prefix_indptr[p+1]-1, sharing prefix_lens[p] tokens
    in the pages of prefix_block_table row p; sequence b's own tokens in block_table row b."""

    k_cache: torch.Tensor
    v_cache: torch.Tensor
    prefix_block_table: torch.Tensor
    prefix_lens: torch.Tensor
    prefix_indptr: torch.Tensor
    block_table: torch.Tensor
    seq_lens: torch.Tensor
    page_size: int

    def concatenated_tables(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(block_table, seq_lens) of the same problem without sharing: each sequence's row
        lists its group's prefix pages, then its own. Exact only when every prefix length is a
        multiple of the page size (a partial prefix page would sit in the middle)."""
        indptr = self.prefix_indptr.tolist()
        plens = self.prefix_lens.tolist()
        group = [p for p in range(len(plens)) for _ in range(indptr[p], indptr[p + 1])]
        rows, lens = [], []
        for b, n in enumerate(self.seq_lens.tolist()):
            pl = plens[group[b]]
            pp = pages_for(pl, self.page_size)
            rows.append(self.prefix_block_table[group[b], :pp].tolist() +
                        self.block_table[b, : pages_for(n, self.page_size)].tolist())
            lens.append(pl + n)
        width = max(1, max(len(r) for r in rows))
        table = torch.zeros((len(rows), width), dtype=torch.int32)
        for b, r in enumerate(rows):
            table[b, : len(r)] = torch.tensor(r, dtype=torch.int32)
        dev = self.block_table.device
        return table.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev)


def random_cascade_problem(
    group_sizes: list[int],
    prefix_lens: list[int],
    seq_lens: list[int],
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    page_size: int,
    dtype: torch.dtype = torch.bfloat16,
    device: str | torch.device = "cuda",
    seed: int = 0,
    poison: float = NAN,
) -> tuple[torch.Tensor, CascadeKV]:
    """A seeded shared-prefix problem: len(group_sizes) groups of consecutive sequences (sizes
    summing to len(seq_lens)), group p's prefix of prefix_lens[p] tokens, and each sequence's
    own seq_lens[b] tokens, all in one shuffled pool with poisoned spare pages
    (random_paged_pool over the prefixes followed by the sequences)."""
    assert len(group_sizes) == len(prefix_lens) and sum(group_sizes) == len(seq_lens)
    groups = len(prefix_lens)
    q_all, kv = random_paged_pool(
        [*prefix_lens, *seq_lens], num_q_heads, num_kv_heads, head_dim, page_size, dtype=dtype, device=device,
        seed=seed, poison=poison,
    )
    dev = kv.block_table.device
    table = kv.block_table
    wp = max(1, max(pages_for(n, page_size) for n in prefix_lens))
    ws = max(1, max(pages_for(n, page_size) for n in seq_lens))
    if table.shape[1] < max(wp, ws):
        table = torch.nn.functional.pad(table, (0, max(wp, ws) - table.shape[1]))
    indptr = [0]
    for g in group_sizes:
        indptr.append(indptr[-1] + g)
    return q_all[groups:].contiguous(), CascadeKV(
        k_cache=kv.k_cache,
        v_cache=kv.v_cache,
        prefix_block_table=table[:groups, :wp].contiguous(),
        prefix_lens=torch.tensor(prefix_lens, dtype=torch.int32, device=dev),
        prefix_indptr=torch.tensor(indptr, dtype=torch.int32, device=dev),
        block_table=table[groups:, :ws].contiguous(),
        seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=dev),
        page_size=page_size,
    )


def quantize_e4m3(cache: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """A [num_pages, page, num_kv_heads, head_dim] cache as e4m3 codes with per-KV-head scales:
    e4m3(x / scale[h]), rounded to nearest-even and saturated to +-448 (NaN poison stays NaN),
    the rounding of the kernels' quantising append."""
    x = cache.float() / scale.float().view(1, 1, -1, 1)
    return torch.where(torch.isnan(x), x, x.clamp(-448.0, 448.0)).to(torch.float8_e4m3fn)


def e4m3_scales(cache: torch.Tensor, margin: float = 1.0) -> torch.Tensor:
    """Per-KV-head scales that map each head's largest finite magnitude to 448 / margin."""
    x = cache.float()
    amax = torch.where(torch.isfinite(x), x.abs(), torch.zeros_like(x)).amax(dim=(0, 1, 3))
    return (amax.clamp_min(1e-12) * margin / 448.0).float().contiguous()
