"""Shared test setup.

Two tiers, as in kernel-lab's suite: CPU tests (oracle vs the golden vectors, host logic,
the C ABI's exports, gloo multi-process paths) run anywhere; ``@pytest.mark.gpu`` tests
run the CUDA kernels on a B200 and compare them with the oracle and the golden vectors.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "kernel-lab_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

HAS_GPU = torch.cuda.is_available()

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DT_NAME = {v: k for k, v in DT.items()}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def tolerance(dtype: torch.dtype) -> dict[str, float]:
    """kernel-lab's per-dtype tolerances (tests/conftest.py:34-39 there)."""
    return {
        torch.float32: {"atol": 1e-4, "rtol": 1e-4},
        torch.float16: {"atol": 2e-3, "rtol": 2e-3},
        torch.bfloat16: {"atol": 1.6e-2, "rtol": 1.6e-2},
    }[dtype]


# The north star's bound: max-abs error vs the fp32-math oracle.
NORTH_STAR_MAX_ABS = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 2e-2}
SIGNIFICAND_BITS = {torch.float32: 24, torch.float16: 11, torch.bfloat16: 8}


def ulp(dtype: torch.dtype, v: np.ndarray) -> np.ndarray:
    """Spacing of `dtype` values at |v|."""
    e = np.floor(np.log2(np.maximum(np.abs(v), 2.0**-126)))
    return 2.0 ** (e - (SIGNIFICAND_BITS[dtype] - 1))


def assert_within_abs_or_ulp(got: torch.Tensor, exact: np.ndarray, dtype: torch.dtype, atol: float | None = None):
    """|got - exact| <= max(atol, one ulp of dtype at |exact|) everywhere, with `exact` the
    unrounded fp32 oracle. atol defaults to the north star's bound. Where |exact| is large
    the two storage values nearest the exact result are more than atol apart, so one ulp
    is the tightest achievable bound there."""
    atol = NORTH_STAR_MAX_ABS[dtype] if atol is None else atol
    g = got.float().cpu().numpy()
    assert np.isfinite(g).all()
    err = np.abs(g - exact)
    bound = np.maximum(atol, ulp(dtype, exact))
    worst = int(np.argmax(err - bound))
    assert (err <= bound).all(), f"err {err.flat[worst]} > bound {bound.flat[worst]} at |y|={abs(exact.flat[worst])}"
    return float(err.max())


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def to_f32_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def golden_to_torch(arr: np.ndarray, dt: str) -> torch.Tensor:
    if dt == "bf16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(arr.copy())


_INDEX = None
_ARRAYS: dict[str, np.lib.npyio.NpzFile] = {}


def golden_index() -> dict:
    global _INDEX
    if _INDEX is None:
        _INDEX = json.loads((GOLDEN / "index.json").read_text())
    return _INDEX


def golden_array(kind: str, key: str) -> np.ndarray:
    if kind not in _ARRAYS:
        _ARRAYS[kind] = np.load(GOLDEN / f"{kind}.npz")
    return _ARRAYS[kind][key]


def decode_case(name: str) -> dict:
    for c in golden_index()["decode"]:
        if c["name"] == name:
            return c
    raise KeyError(name)


def build_decode_case(case: dict, device: str = "cpu", poison: float = float("nan")):
    """Inputs of a golden decode case, rebuilt with this repository's fixture builder."""
    from kernel_lab.kv_cache import random_decode_problem

    return random_decode_problem(
        case["lens"], case["hq"], case["hkv"], case["d"], case["p"], dtype=DT[case["dt"]], device=device,
        seed=0, poison=poison,
    )


def make_rms_inputs(shape, dtype, seed=0):
    """kernel-lab's RMSNorm input protocol (tests/test_rmsnorm.py:14-19 there)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g).to(dtype=dtype)
    r = torch.randn(*shape, generator=g).to(dtype=dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype=dtype)
    return x, r, w
