"""Timed CPU runs of the oracle (TEST / BASELINE INFRASTRUCTURE ONLY).

Used by ``bench.py`` for its ``cpu_baseline`` figure and its ``--impl reference`` arm:
kernel-lab's reference path is PyTorch-on-CPU Python (kernel_lab/reference.py:33-68),
which cannot travel to the GPU box, so its NumPy restatement (``oracle.oracle``) is timed
instead, on the box's host cores. Work is spread over a process pool (``spawn`` start
method, never ``fork``: the parent may already hold a CUDA context), one sequence per
task, so every core is busy; each worker builds its own seeded sample once, so the timed
region contains only the oracle's arithmetic and the task dispatch.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import time
from concurrent.futures import ProcessPoolExecutor

import numpy as np

_STATE: dict = {}


def _worker_init(kind: str, spec: dict, seed: int) -> None:
    # One BLAS thread per process: the pool already occupies every core.
    from threadpoolctl import threadpool_limits

    _STATE["blas_limit"] = threadpool_limits(1)
    from oracle import oracle

    rng = np.random.default_rng(seed + os.getpid())
    dt = spec["dtype"]
    if kind == "decode":
        ctx, hq, hkv, d, page = spec["ctx"], spec["hq"], spec["hkv"], spec["d"], spec["page"]
        pages = (ctx + page - 1) // page
        order = rng.permutation(pages + 3).astype(np.int32)
        rnd = lambda *s: oracle.round_to(rng.standard_normal(s, dtype=np.float32), dt)  # noqa: E731
        k = np.full((pages + 3, page, hkv, d), np.nan, np.float32)
        v = np.full_like(k, np.nan)
        k[order[:pages]] = rnd(pages, page, hkv, d)
        v[order[:pages]] = rnd(pages, page, hkv, d)
        _STATE.update(q=rnd(1, hq, d), k=k, v=v, bt=order[None, :pages].copy(), lens=np.array([ctx], np.int32))
    else:
        rows, hidden = spec["rows"], spec["hidden"]
        _STATE.update(
            x=oracle.round_to(rng.standard_normal((rows, hidden), dtype=np.float32), dt),
            r=oracle.round_to(rng.standard_normal((rows, hidden), dtype=np.float32), dt),
            w=oracle.round_to(1 + 0.1 * rng.standard_normal(hidden, dtype=np.float32), dt),
        )
    _STATE["kind"], _STATE["dtype"] = kind, dt


def _worker_step(_: int) -> float:
    from oracle import oracle

    t0 = time.perf_counter()
    s = _STATE
    if s["kind"] == "decode":
        oracle.paged_decode_attention(s["q"], s["k"], s["v"], s["bt"], s["lens"], None, s["dtype"])
    else:
        oracle.fused_add_rms_norm(s["x"], s["r"], s["w"], 1e-5, s["dtype"])
    return time.perf_counter() - t0


class CpuOracleRunner:
    """A pool of `workers` processes; one step = every worker runs the oracle on its sample unit.

    decode: a unit is one sequence (`ctx` tokens, all heads); rmsnorm: `rows` x `hidden`.
    """

    def __init__(self, kind: str, spec: dict, workers: int | None = None, seed: int = 0):
        self.kind, self.spec = kind, spec
        self.workers = workers or os.cpu_count() or 1
        ctx = mp.get_context("spawn")
        self.pool = ProcessPoolExecutor(self.workers, mp_context=ctx, initializer=_worker_init,
                                        initargs=(kind, spec, seed))

    def step(self) -> float:
        """Run one step on all workers; return its wall time in seconds."""
        t0 = time.perf_counter()
        list(self.pool.map(_worker_step, range(self.workers)))
        return time.perf_counter() - t0

    def close(self) -> None:
        self.pool.shutdown(wait=True, cancel_futures=True)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
