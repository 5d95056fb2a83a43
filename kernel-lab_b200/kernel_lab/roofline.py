"""Roofline bookkeeping for the two hot paths: algorithmic bytes and FLOPs, and B200 peaks.

The byte model is kernel-lab's (kernel_lab/bench/roofline.py:57-84): every input read
once, every output written once; for decode, K and V once plus q and out once (block
table and seq_lens not counted). Both kernels are HBM-bound, so "% of peak bandwidth"
is the efficiency figure.

Peaks: the measured copy bandwidth and bf16 GEMM rate in ``MEASURED_PEAKS.json`` at the
repository root when present (written per GPU pool), else the pool's fallback figures,
and the B200 spec sheet for context.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]

B200_SPEC_HBM_GBPS = 8000.0  # HBM3e spec (DGX); the HGX figure is 7.7 TB/s
B200_SPEC_BF16_TFLOPS = 2250.0  # dense
FALLBACK_HBM_GBPS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


@dataclass(frozen=True)
class Work:
    bytes: float
    flops: float

    @property
    def intensity(self) -> float:
        return self.flops / self.bytes


def rms_norm_work(rows: int, hidden: int, elem_bytes: int, fused_residual: bool) -> Work:
    """x in and out out (plus residual in and out when fused), plus the weight once."""
    tensors = 4 if fused_residual else 2
    return Work(
        bytes=rows * hidden * elem_bytes * tensors + hidden * elem_bytes,
        flops=rows * hidden * (5 if fused_residual else 4),
    )


def decode_attention_work(
    seq_lens: list[int], num_q_heads: int, num_kv_heads: int, head_dim: int, elem_bytes: int,
    kv_elem_bytes: int | None = None,
) -> Work:
    """K and V of every cached token once, q read and out written once; 4*D FLOPs per (head, token).
    ``kv_elem_bytes`` (default ``elem_bytes``) is the cache's element size: 1 for an e4m3 cache."""
    tokens = sum(max(int(n), 0) for n in seq_lens)
    kv = 2 * tokens * num_kv_heads * head_dim * (elem_bytes if kv_elem_bytes is None else kv_elem_bytes)
    q_out = 2 * len(seq_lens) * num_q_heads * head_dim * elem_bytes
    return Work(bytes=kv + q_out, flops=4 * tokens * num_q_heads * head_dim)


@dataclass(frozen=True)
class Peaks:
    hbm_gbps: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    source: str  # "measured" or "fallback"


def measured_peaks(path: Path | None = None) -> Peaks:
    p = path or REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return Peaks(
            float(d["hbm_gbs"]),
            float(d["bf16_tflops"]),
            float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
            "measured",
        )
    except (OSError, KeyError, ValueError):
        return Peaks(FALLBACK_HBM_GBPS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback")
