"""NumPy restatement of kernel-lab's fp32 reference math (TEST INFRASTRUCTURE ONLY).

This module is the checker for the CUDA kernels and the timed CPU baseline in
``bench.py``. It is not part of the product and is never called by it.

Parity is pinned: ``tests/test_oracle.py`` checks every function here against the
golden vectors in ``tests/golden/``, which ``tests/golden/make_golden.py``
produced by running the reference's own ``kernel_lab/reference.py`` and
``kernel_lab/kv_cache.py`` (PyTorch, CPU) on seeded inputs.

Arrays are NumPy float32 holding values that are exactly representable in the
storage dtype ("f32", "f16" or "bf16"), because NumPy has no bfloat16. The
functions round to the storage dtype at the same points as the reference: the
residual stream after the add, and every output (kernel_lab/reference.py:1-6).
"""

from __future__ import annotations

import numpy as np

DTYPES = ("f32", "f16", "bf16")
ELEM_BYTES = {"f32": 4, "f16": 2, "bf16": 2}
LOG2E = 1.4426950408889634


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` with round-to-nearest-even; return float32.

    fp16 uses NumPy's IEEE half. bf16 keeps the top 16 bits of the float32 pattern
    after adding half an ulp plus the tie-to-even bit; NaN stays NaN.
    """
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype != "bf16":
        raise ValueError(f"unknown dtype {dtype!r}")
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = np.float32("nan")
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bfloat16 bit patterns (round to nearest even)."""
    return (round_to(x, "bf16").view(np.uint32) >> 16).astype(np.uint16)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6, dtype: str = "f32") -> np.ndarray:
    """y = x / sqrt(mean(x^2) + eps) * weight over the last axis, fp32 math, rounded to dtype.

    Follows kernel_lab/reference.py:13-17: the product is formed as (x * rstd) * w.
    """
    xf = np.asarray(x, dtype=np.float32)
    ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    rstd = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return round_to((xf * rstd) * np.asarray(weight, dtype=np.float32), dtype)


def fused_add_rms_norm(
    x: np.ndarray, residual: np.ndarray, weight: np.ndarray, eps: float = 1e-6, dtype: str = "f32"
) -> tuple[np.ndarray, np.ndarray]:
    """Pre-norm step: new_residual = dtype(x + residual); out = rms_norm(new_residual).

    Follows kernel_lab/reference.py:20-30. The sum is formed in fp32 and rounded
    once to the storage dtype, so the residual output is bit-exact.
    """
    new_residual = round_to(np.asarray(x, np.float32) + np.asarray(residual, np.float32), dtype)
    return rms_norm(new_residual, weight, eps, dtype), new_residual


def paged_decode_attention(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_table: np.ndarray,
    seq_lens: np.ndarray,
    scale: float | None = None,
    dtype: str = "f32",
) -> np.ndarray:
    """Single-token GQA decode attention over a paged KV cache (NHD layout), fp32 math.

    Follows kernel_lab/reference.py:33-68:
        q            [batch, num_q_heads, head_dim]
        k/v_cache    [num_pages, page_size, num_kv_heads, head_dim]
        block_table  [batch, >= ceil(len/page_size)] int32 page ids, in order
        seq_lens     [batch] int32
    Only the first ceil(len / page_size) block-table entries of a row are read,
    so spare (poisoned) pages and padding never enter the result. A sequence of
    length 0 yields zeros, as the reference's empty einsum does.
    """
    q = np.asarray(q, dtype=np.float32)
    batch, _, head_dim = q.shape
    page_size = k_cache.shape[1]
    scale = head_dim**-0.5 if scale is None else scale
    out = np.zeros_like(q)
    for b in range(batch):
        length = max(int(seq_lens[b]), 0)
        if length == 0:
            continue
        pages = np.asarray(block_table[b, : (length + page_size - 1) // page_size], dtype=np.int64)
        k = _token_rows(k_cache, pages, length)  # [L, Hkv, D]
        v = _token_rows(v_cache, pages, length)
        out[b] = _attend(q[b], k, v, scale)
    return round_to(out, dtype)


def _attend(qb: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """softmax(scale * q . K^T) V for one sequence, fp32 (kernel_lab/reference.py:62-67): qb [Hq, D],
    k and v [L, Hkv, D], query head h attending with KV head h // (Hq / Hkv)."""
    num_q_heads, head_dim = qb.shape
    num_kv_heads = k.shape[1]
    q3 = qb.reshape(num_kv_heads, num_q_heads // num_kv_heads, head_dim)
    scores = np.einsum("hgd,lhd->hgl", q3, k, optimize=True) * np.float32(scale)  # [Hkv, G, L]
    scores -= scores.max(axis=-1, keepdims=True)
    probs = np.exp(scores, dtype=np.float32)
    probs /= probs.sum(axis=-1, keepdims=True, dtype=np.float32)
    return np.einsum("hgl,lhd->hgd", probs, v, optimize=True).reshape(num_q_heads, head_dim)


def _token_rows(cache: np.ndarray, pages: np.ndarray, length: int) -> np.ndarray:
    """The first `length` token rows [L, Hkv, D] (fp32) of the pages `pages` of a paged cache: a
    view when the pages are consecutive, else a gather."""
    _, page_size, num_kv_heads, head_dim = cache.shape
    if len(pages) and pages[0] >= 0 and np.array_equal(pages, np.arange(pages[0], pages[0] + len(pages))):
        rows = cache[pages[0] : pages[0] + len(pages)]
    else:
        rows = cache[pages]
    return np.asarray(rows, np.float32).reshape(-1, num_kv_heads, head_dim)[:length]


def _gather_tokens(cache: np.ndarray, pages_row: np.ndarray, length: int) -> np.ndarray:
    """First ``length`` token rows [L, Hkv, D] of the pages listed in ``pages_row``."""
    page_size = cache.shape[1]
    pages = np.asarray(pages_row[: (length + page_size - 1) // page_size], dtype=np.int64)
    return np.asarray(cache[pages], np.float32).reshape(-1, cache.shape[2], cache.shape[3])[:length]


def paged_decode_attention_cascade(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    prefix_block_table: np.ndarray,
    prefix_lens: np.ndarray,
    prefix_indptr: np.ndarray,
    block_table: np.ndarray,
    seq_lens: np.ndarray,
    scale: float | None = None,
    dtype: str = "f32",
) -> np.ndarray:
    """Shared-prefix (cascade) decode: sequence b of group p (prefix_indptr[p] <= b <
    prefix_indptr[p+1]) attends to the prefix_lens[p] tokens of row p of prefix_block_table
    followed by its own seq_lens[b] tokens (row b of block_table). kernel-lab has no cascade
    (its design notes name it as FlashInfer's addition, docs/design.md:96-102); the result is
    kernel-lab's reference decode math (kernel_lab/reference.py:33-68) over that concatenated
    token list. A group table that does not partition the batch (first entry 0, non-decreasing,
    last entry batch) makes the prefixes ignored, as the kernel does.
    """
    q = np.asarray(q, dtype=np.float32)
    batch, _, head_dim = q.shape
    scale = head_dim**-0.5 if scale is None else scale
    indptr = np.asarray(prefix_indptr, dtype=np.int64)
    groups = len(prefix_lens)
    valid = groups > 0 and indptr[0] == 0 and indptr[groups] == batch and bool(np.all(np.diff(indptr) >= 0))
    prefix_cap = prefix_block_table.shape[1] * k_cache.shape[1]
    own_cap = block_table.shape[1] * k_cache.shape[1]
    out = np.zeros_like(q)
    for b in range(batch):
        ks, vs = [], []
        if valid:
            p = int(np.searchsorted(indptr, b, side="right")) - 1
            plen = min(max(int(prefix_lens[p]), 0), prefix_cap)
            if plen > 0:
                ks.append(_gather_tokens(k_cache, prefix_block_table[p], plen))
                vs.append(_gather_tokens(v_cache, prefix_block_table[p], plen))
        length = min(max(int(seq_lens[b]), 0), own_cap)
        if length > 0:
            ks.append(_gather_tokens(k_cache, block_table[b], length))
            vs.append(_gather_tokens(v_cache, block_table[b], length))
        if not ks:
            continue
        out[b] = _attend(q[b], np.concatenate(ks), np.concatenate(vs), scale)
    return round_to(out, dtype)


KL_STATUS_BAD_PAGE = 1
KL_STATUS_BAD_PREFIX_GROUPS = 8

# ---------------------------------------------------------------- e4m3 (float8 "fn": no infinities)
#
# The FP8 KV cache of kernel-lab's roadmap (README.md:98) stores K and V as e4m3 with one
# scale per KV head: stored = e4m3(x / scale), read = e4m3 value * scale. e4m3: 1 sign bit,
# 4 exponent bits (bias 7), 3 mantissa bits; subnormals below 2**-6; S.1111.111 is NaN;
# largest finite 448. Encoding rounds to nearest-even and saturates to +-448 (the cast that
# the CUDA fp8 conversion performs with its saturate-finite mode). These are restatements
# of the format's published definition; tests pin them against torch.float8_e4m3fn.


def _e4m3_table() -> np.ndarray:
    b = np.arange(256, dtype=np.int64)
    sign = np.where(b >> 7, -1.0, 1.0)
    e = (b >> 3) & 15
    m = (b & 7).astype(np.float64)
    mag = np.where(e == 0, m / 8.0 * 2.0**-6, (1.0 + m / 8.0) * 2.0 ** (e - 7))
    val = sign * mag
    val[(e == 15) & ((b & 7) == 7)] = np.nan
    return val.astype(np.float32)


E4M3_VALUES = _e4m3_table()


def e4m3_decode(bytes_: np.ndarray) -> np.ndarray:
    """uint8 e4m3 codes -> float32 values."""
    return E4M3_VALUES[np.asarray(bytes_, dtype=np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> uint8 e4m3 codes: round to nearest-even, saturate to +-448, NaN stays NaN."""
    x = np.asarray(x, dtype=np.float32)
    a = np.where(np.isnan(x), 0.0, np.abs(x).astype(np.float64))  # NaN is coded at the end
    e = np.clip(np.floor(np.log2(np.maximum(a, 2.0**-12))), -6, 8)
    step = 2.0 ** (e - 3)
    r = np.minimum(np.rint(a / step) * step, 448.0)
    # value -> code: exponent field and mantissa from the rounded magnitude
    re = np.where(r >= 2.0**-6, np.floor(np.log2(np.maximum(r, 2.0**-6))), -7)
    mant = np.where(re >= -6, np.rint((r / 2.0**re - 1.0) * 8.0), np.rint(r / 2.0**-9))
    exp_field = np.where(re >= -6, re + 7, 0)
    code = (exp_field.astype(np.int64) << 3) | mant.astype(np.int64)
    code = np.where(np.signbit(x), code | 0x80, code)
    code = np.where(np.isnan(x), 0x7F, code)
    return code.astype(np.uint8)


def paged_decode_attention_fp8(
    q: np.ndarray,
    k_codes: np.ndarray,
    v_codes: np.ndarray,
    k_scale: np.ndarray,
    v_scale: np.ndarray,
    block_table: np.ndarray,
    seq_lens: np.ndarray,
    scale: float | None = None,
    dtype: str = "f32",
) -> np.ndarray:
    """Decode attention over an e4m3 cache: dequantise (code value * per-KV-head scale), then
    kernel-lab's fp32 reference math (paged_decode_attention above)."""
    k = e4m3_decode(k_codes) * np.asarray(k_scale, np.float32)[None, None, :, None]
    v = e4m3_decode(v_codes) * np.asarray(v_scale, np.float32)[None, None, :, None]
    return paged_decode_attention(q, k, v, block_table, seq_lens, scale, dtype)


def paged_kv_append_fp8(
    k_codes: np.ndarray,
    v_codes: np.ndarray,
    k_new: np.ndarray,
    v_new: np.ndarray,
    k_scale: np.ndarray,
    v_scale: np.ndarray,
    block_table: np.ndarray,
    positions: np.ndarray,
) -> tuple[np.ndarray, np.ndarray, int]:
    """paged_kv_append into an e4m3 cache: each new row is quantised per KV head,
    e4m3(x / scale) with the division done in float32, then scattered like paged_kv_append."""
    ks = np.asarray(k_scale, np.float32)[None, :, None]
    vs = np.asarray(v_scale, np.float32)[None, :, None]
    hkv, d = k_codes.shape[2], k_codes.shape[3]
    kq = e4m3_encode((np.asarray(k_new, np.float32).reshape(-1, hkv, d) / ks).astype(np.float32))
    vq = e4m3_encode((np.asarray(v_new, np.float32).reshape(-1, hkv, d) / vs).astype(np.float32))
    return paged_kv_append(k_codes, v_codes, kq, vq, block_table, positions)


def paged_kv_append(
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    k_new: np.ndarray,
    v_new: np.ndarray,
    block_table: np.ndarray,
    positions: np.ndarray,
    max_pages: int | None = None,
) -> tuple[np.ndarray, np.ndarray, int]:
    """Write token ``positions[b]`` of every sequence into its page of the NHD pool.

    The pool layout is kernel-lab's (csrc/kernel_lab.h:21-26: ``[num_pages, page_size,
    num_kv_heads, head_dim]``): token t of sequence b lives at page ``block_table[b, t // P]``,
    slot ``t % P``, which is how kernel-lab's fixtures fill it (kernel_lab/kv_cache.py:66-72)
    and how its decode reads it (csrc/paged_attention.cu:68-70). kernel-lab has no append op;
    this restates that layout as a scatter. Negative positions skip their sequence; a position
    past ``max_pages * P`` or a page id outside the pool skips it and sets the bad-page bit.
    Returns new caches (the inputs are not modified) and the status bits.
    """
    k = np.array(k_cache, copy=True)
    v = np.array(v_cache, copy=True)
    num_pages, page_size = k.shape[0], k.shape[1]
    width = block_table.shape[1] if max_pages is None else max_pages
    status = 0
    for b, pos in enumerate(np.asarray(positions).tolist()):
        if pos < 0:
            continue
        pidx = pos // page_size
        page = int(block_table[b, pidx]) if pidx < width else -1
        if page < 0 or page >= num_pages:
            status |= KL_STATUS_BAD_PAGE
            continue
        k[page, pos % page_size] = np.asarray(k_new[b]).reshape(k.shape[2:])
        v[page, pos % page_size] = np.asarray(v_new[b]).reshape(v.shape[2:])
    return k, v, status


def decode_bytes(seq_lens, num_q_heads: int, num_kv_heads: int, head_dim: int, elem_bytes: int) -> int:
    """Algorithmic HBM bytes of one decode call: K and V read once, q read and out written once.

    Same count as kernel_lab/bench/roofline.py:76-84; block table and seq_lens are not counted.
    """
    tokens = int(np.sum(np.maximum(np.asarray(seq_lens, dtype=np.int64), 0)))
    return 2 * tokens * num_kv_heads * head_dim * elem_bytes + 2 * len(seq_lens) * num_q_heads * head_dim * elem_bytes
