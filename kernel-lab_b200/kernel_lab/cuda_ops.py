"""Python wrappers for the CUDA kernels (torch.ops.kernel_lab.*).

Same API as kernel-lab's ``kernel_lab/cuda_ops.py:11-61`` (``available``,
``why_unavailable``, ``rms_norm``, ``fused_add_rms_norm``, ``paged_decode_attention``),
plus ``num_splits`` on ``paged_decode_attention`` and ``decode_status``. There is no
fallback: if the extension is not built these functions raise RuntimeError.
"""

from __future__ import annotations

import torch

try:
    from kernel_lab import _C  # registers torch.ops.kernel_lab

    _LOADED = True
    _LOAD_ERROR = ""
except ImportError as exc:  # not built
    _LOADED = False
    _LOAD_ERROR = str(exc)


def available() -> bool:
    return _LOADED and torch.cuda.is_available()


def why_unavailable() -> str:
    if not _LOADED:
        return f"CUDA extension not built ({_LOAD_ERROR}); run `python kernel-lab_b200/build.py`"
    return "no CUDA device"


def _require() -> None:
    if not _LOADED:
        raise RuntimeError(f"kernel_lab: {why_unavailable()}")


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    _require()
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    torch.ops.kernel_lab.rms_norm(out, x, weight, eps)
    return out


def fused_add_rms_norm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6
) -> tuple[torch.Tensor, torch.Tensor]:
    """Functional form: returns (out, new_residual) and leaves ``residual`` untouched.
    Call torch.ops.kernel_lab.fused_add_rms_norm directly to update in place."""
    _require()
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    new_residual = residual.contiguous().clone()
    torch.ops.kernel_lab.fused_add_rms_norm(out, x, new_residual, weight, eps)
    return out, new_residual


def paged_decode_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    num_splits: int | None = None,
) -> torch.Tensor:
    """Decode attention over a paged cache. ``num_splits=None`` uses the load-balanced
    planner; an integer forces that many KV splits per sequence (Triton semantics)."""
    _require()
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    out = torch.empty_like(q)
    if num_splits is None:
        torch.ops.kernel_lab.paged_decode_attention(out, q.contiguous(), k_cache, v_cache, block_table, seq_lens, scale)
    else:
        torch.ops.kernel_lab.paged_decode_attention_splits(
            out, q.contiguous(), k_cache, v_cache, block_table, seq_lens, scale, int(num_splits)
        )
    return out


def paged_kv_append(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    block_table: torch.Tensor,
    positions: torch.Tensor,
) -> None:
    """Write each sequence's new token's K/V rows ([batch, num_kv_heads, head_dim], rows may be a
    strided view) into its pages at token index ``positions[b]`` (in place; negative skips).
    Page ids outside the pool are skipped and reported by :func:`decode_status`."""
    _require()
    torch.ops.kernel_lab.paged_kv_append(k_cache, v_cache, k_new, v_new, block_table, positions)


def paged_decode_attention_fp8(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
) -> torch.Tensor:
    """Decode attention over an e4m3 KV cache (torch.float8_e4m3fn) with per-KV-head float32
    scales: K = code * k_scale[h], V = code * v_scale[h]. q is fp16 or bf16."""
    _require()
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    out = torch.empty_like(q)
    torch.ops.kernel_lab.paged_decode_attention_fp8(
        out, q.contiguous(), k_cache, v_cache, k_scale, v_scale, block_table, seq_lens, scale
    )
    return out


def paged_kv_append_fp8(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    positions: torch.Tensor,
) -> None:
    """paged_kv_append into an e4m3 cache: rows are quantised per KV head as
    e4m3(x / scale) (round to nearest-even, saturating to +-448)."""
    _require()
    torch.ops.kernel_lab.paged_kv_append_fp8(k_cache, v_cache, k_new, v_new, k_scale, v_scale, block_table, positions)


def paged_decode_attention_cascade(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    prefix_block_table: torch.Tensor,
    prefix_lens: torch.Tensor,
    prefix_indptr: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
) -> torch.Tensor:
    """Shared-prefix (cascade) decode: the sequences of group p, ``prefix_indptr[p]`` up to
    ``prefix_indptr[p + 1]``, attend to the ``prefix_lens[p]`` tokens held in the pages of row p
    of ``prefix_block_table`` and then to their own ``seq_lens[b]`` tokens (``block_table`` row b).
    A prefix's pages are read once per block of its group's sequences, not once per sequence.
    With ``k_scale`` / ``v_scale`` the caches are e4m3 (torch.float8_e4m3fn)."""
    _require()
    out = torch.empty_like(q)
    torch.ops.kernel_lab.paged_decode_attention_cascade(
        out, q, k_cache, v_cache, prefix_block_table, prefix_lens, prefix_indptr, block_table, seq_lens,
        q.shape[-1] ** -0.5 if scale is None else scale, k_scale, v_scale,
    )
    return out


def decode_status(clear: bool = False) -> int:
    """KL_STATUS_* bits left by decode and append calls on the current device and stream
    (synchronises)."""
    _require()
    return int(_C.decode_status(clear))
