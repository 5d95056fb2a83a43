"""Benchmark of the paged-decode hot path (and fused add + RMSNorm) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}] [--workload ...]

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N

Workload (default ``decode``): kernel-lab's headline, paged decode attention with Llama-3-8B
heads (32 query / 8 KV, head_dim 128, 16-token pages), bf16, batch 64, context 4096,
shuffled pages, NaN-poisoned spare pages. A step is one decode call. At N GPUs the batch grows
to 64*N and the KV heads are sharded N ways (tensor parallel): rank r holds KV heads
[r*8/N, (r+1)*8/N) of every sequence and their query heads, so every GPU streams the same
1.07 GB of KV per step (weak scaling), and the decode kernel itself stores its heads into every
rank's [64*N, 32, 128] output over NVLink (one launch per step does attention and gather). The
default line at N=1 also carries ``grid`` (config 3's six batch x context cells) and
``secondary`` (fused add + RMSNorm, 4096 x 8192 bf16).

Other workloads: ``decode_seq`` (the headline with the batch split by sequence at N > 1: no
exchange at all); ``decode_fp8`` (the headline over an e4m3 KV cache, per-KV-head scales, KV
bytes counted at one per element); ``decode70b`` (Llama-3-70B heads 64/8, batch 256, context
8192, total work fixed across N: strong scaling over the same KV-head shards and fused gather);
``cascade`` (64 sequences per GPU sharing a 4096-token prefix, 512 own tokens each); ``ragged``
(config 4: batch 128, lengths uniform in [1, 32768] plus 16k-1, 16k, 16k+1, in the MQA 32/1,
GQA 32/8 and MHA 32/32 layouts, one GPU); ``rmsnorm`` (fused add + RMSNorm, 4096 x 8192 bf16).

One JSON line on rank 0: value = aggregate algorithmic HBM GB/s (K+V read once, q and
out once: kernel-lab's byte model) over the max-over-ranks device time; ``roofline`` for
the decode kernel (its own CUDA-event time); ``e2e`` through the public API with pinned host
inputs copied in and the output copied out every step; ``cpu_baseline`` = the oracle
(NumPy restatement of kernel-lab's PyTorch CPU reference) on this host's cores.
``--impl reference`` times that CPU path alone (kernel-lab's own implementation of the
path is PyTorch-on-CPU; its restatement stands in for it on the GPU box).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path[:0] = [str(REPO), str(REPO / "kernel-lab_b200")]

METRIC = "paged decode attn % of B200 peak HBM BW (Llama-3-8B GQA bs64 ctx4096); us/call"
RMS_METRIC = "fused add+RMSNorm % of B200 peak HBM BW (4096 tokens x 8192 hidden, bf16); us/call"
FP8_METRIC = "paged decode attn, e4m3 KV cache, algorithmic HBM GB/s (Llama-3-8B GQA bs64 ctx4096); us/call"
CASCADE_METRIC = ("cascade (shared-prefix) decode, unique KV bytes GB/s (Llama-3-8B GQA, 64 sequences sharing a "
                  "4096-token prefix + 512 own tokens each); us/call")
RAGGED_METRIC = ("ragged-batch paged decode attn, algorithmic HBM GB/s over MQA 32/1, GQA 32/8 and MHA 32/32 "
                 "(batch 128, lengths U[1, 32768]); us/call")
L2_NOTE = "inputs larger than L2 (no flush needed)"
L2_BYTES = 126 * 1024 * 1024


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "ours", "reference"], default="b200")
    ap.add_argument("--workload", choices=["decode", "decode_seq", "decode_fp8", "decode70b", "cascade", "ragged",
                                           "rmsnorm"], default="decode")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the grid and secondary objects of the default line")
    ap.add_argument("--batch", type=int, help="override the workload's batch (per GPU for weak scaling)")
    ap.add_argument("--ctx", type=int, help="override the workload's context length")
    ap.add_argument("--heads", help="override the decode workload's heads as HQ/HKV (e.g. 4/1: one GPU's share "
                                    "of Llama-3-8B's heads sharded 8 ways)")
    return ap.parse_args()


def ragged_lens(batch: int = 128, seed: int = 4) -> list[int]:
    """Config 4's lengths: uniform in [1, 32768] from a seed, with 16k - 1, 16k and 16k + 1."""
    from kernel_lab.kv_cache import config4_lengths

    return config4_lengths(batch, seed)


RAGGED_LAYOUTS = {"mqa": (32, 1), "gqa": (32, 8), "mha": (32, 32)}


def workload_spec(name: str, world: int) -> dict:
    if name == "decode":
        if world == 1:
            return dict(kind="decode", batch=64, ctx=4096, hq=32, hkv=8, d=128, page=16, scaling="weak",
                        layout="single",
                        desc="paged decode, Llama-3-8B heads 32/8/128, page 16, bf16, batch 64, ctx 4096")
        # KV heads sharded N ways, batch 64 per GPU's worth of KV, heads gathered by the kernel.
        return dict(kind="decode", batch=64 * world, ctx=4096, hq=32, hkv=8, d=128, page=16, scaling="weak",
                    layout="kv_heads",
                    desc=f"paged decode, Llama-3-8B heads 32/8/128 sharded {world} ways by KV head, page 16, bf16, "
                         f"batch {64 * world} (64 per GPU of KV), ctx 4096, heads gathered over NVLink by the kernel")
    if name == "decode_seq":
        # Sequences are independent: each rank decodes its own 64 with every head, no exchange.
        return dict(kind="decode", batch=64 * world, ctx=4096, hq=32, hkv=8, d=128, page=16, scaling="weak",
                    layout="sequences",
                    desc="paged decode, Llama-3-8B heads 32/8/128, page 16, bf16, batch 64/GPU split by sequence, "
                         "ctx 4096")
    if name == "decode_fp8":
        # The headline with an e4m3 KV cache (per-KV-head scales): half the KV bytes per token.
        return dict(kind="decode", batch=64 * world, ctx=4096, hq=32, hkv=8, d=128, page=16, scaling="weak",
                    layout="sequences", kv8=True,
                    desc="paged decode, e4m3 KV cache, Llama-3-8B heads 32/8/128, page 16, bf16 q/out, "
                         "batch 64/GPU, ctx 4096")
    if name == "cascade":
        # Shared prefix: each GPU's 64 sequences share one 4096-token prefix and own 512 tokens.
        return dict(kind="decode", batch=64 * world, ctx=512, prefix=4096, hq=32, hkv=8, d=128, page=16,
                    scaling="weak", layout="sequences", cascade=True,
                    desc="cascade decode, Llama-3-8B heads 32/8/128, page 16, bf16, batch 64/GPU sharing a "
                         "4096-token prefix, 512 own tokens each")
    if name == "decode70b":
        # Tensor-parallel layout: KV heads sharded, heads gathered by the kernel; total work fixed.
        return dict(kind="decode", batch=256, ctx=8192, hq=64, hkv=8, d=128, page=16, scaling="strong",
                    layout="kv_heads",
                    desc="paged decode, Llama-3-70B heads 64/8/128, page 16, bf16, batch 256, ctx 8192")
    if name == "ragged":
        return dict(kind="ragged", batch=128, d=128, page=16, scaling="weak", layout="single",
                    desc="ragged paged decode, batch 128, lengths U[1, 32768] + 16k-1/16k/16k+1 (seed 4), "
                         "MQA 32/1, GQA 32/8, MHA 32/32 heads of 128, page 16, bf16")
    return dict(kind="rmsnorm", rows=4096, hidden=8192, scaling="weak",
                desc="fused residual-add + RMSNorm, 4096 x 8192 bf16, eps 1e-5")


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """Polls NVML (SM clock, clock-event reasons) on a side thread, every `period` seconds.

    NVML is initialised once per process by `ClockSampler.init`, before the problem is built and
    warmed up: initialising it enumerates every GPU of the node, and done at the start of a timed
    region it stalled the multi-GPU step for milliseconds (8 GPUs: 251 us per step against 209 us;
    an `nvidia-smi` process polling alongside slowed the 2-GPU step tenfold). One poll is taken
    before the region; the side thread starts polling only once the host has enqueued every timed
    step (`launched`), so the polls fall while the GPU works through the region and never meet
    the launch burst. On one GPU such polls cost nothing measurable. On several they still stall
    the synchronised step (2 GPUs: 174 us unpolled, 187-204 us with two polls in the region), so
    multi-GPU runs poll rank 0's GPU only, every 20 ms, in a repeat of the timed steps."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }
    _nvml = None
    _handles: dict = {}

    @classmethod
    def init(cls, device_index: int) -> None:
        """Initialises NVML and this GPU's handle (once; no clocks are reported if NVML is absent)."""
        if device_index in cls._handles:
            return
        try:
            import pynvml

            if cls._nvml is None:
                pynvml.nvmlInit()
                cls._nvml = pynvml
            h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            cls._handles[device_index] = (h, pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:
            pass

    def __init__(self, device_index: int, period: float = 0.005, enabled: bool = True):
        self.samples: list[tuple[int, int]] = []  # taken while the GPU runs the timed steps
        self.edge_samples: list[tuple[int, int]] = []  # just before and just after
        self.max_mhz = None
        self.period = period
        self._stop = threading.Event()
        self._nvml = None
        if not enabled or device_index not in ClockSampler._handles:
            return
        self._nvml = ClockSampler._nvml
        self._h, self.max_mhz = ClockSampler._handles[device_index]

    def _sample(self, edge: bool = False):
        n = self._nvml
        mhz = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
        reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        (self.edge_samples if edge else self.samples).append((mhz, reasons))

    def _run(self):
        self._go.wait()
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self._stop.wait(self.period)

    def launched(self):
        """The host has enqueued the timed steps: poll from now on, while the GPU works through
        them. No poll overlaps the burst of launches (a poll that did stalled the multi-GPU step
        by ~15 us per step over 200 steps at 2 GPUs)."""
        if self._nvml:
            self._go.set()

    def __enter__(self):
        if self._nvml:
            self._sample(edge=True)  # before the region
            self._go = threading.Event()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._nvml:
            self._stop.set()
            self._go.set()
            self._t.join()
            self._sample(edge=True)  # after the region

    def summary(self) -> dict | None:
        """Median SM clock and the union of clock-event reasons of the polls taken while the GPU ran
        the timed steps (the two edge polls only if the region was too short for any)."""
        used = self.samples or self.edge_samples
        if not self._nvml or not used:
            return None
        reasons = 0
        for _, r in used:
            reasons |= r
        names = sorted(k for k, bit in self.REASONS.items() if reasons & bit and k != "gpu_idle")
        return {
            "sm_mhz": statistics.median(m for m, _ in used),
            "sm_max_mhz": self.max_mhz,
            "reasons": names,
            "samples": len(used),
            "in_region": bool(self.samples),
        }


# ----------------------------------------------------------------------------- CPU side


def cpu_unit_spec(spec: dict) -> dict:
    """The decode workload a CPU sample unit comes from: one sequence of the workload's shape (a
    ragged batch: a GQA sequence of its mean length, 16384)."""
    if spec["kind"] == "ragged":
        return dict(spec, kind="decode", ctx=16384, hq=32, hkv=8)
    return spec


def cpu_measure(kind: str, spec: dict, seconds: float, dtype: str = "bf16", warmup: int = 1) -> dict:
    """The oracle on this host: whole sample units per step, until `seconds` of timed work."""
    from oracle.oracle import decode_bytes
    from oracle.timing import CpuOracleRunner

    spec = cpu_unit_spec(spec)
    kind = spec["kind"] if kind != "rmsnorm" else kind
    if kind == "decode":
        unit = dict(ctx=spec["ctx"], hq=spec["hq"] // spec.get("tp", 1), hkv=spec["hkv"] // spec.get("tp", 1),
                    d=spec["d"], page=spec["page"], dtype=dtype)
        unit_bytes = decode_bytes([unit["ctx"]], unit["hq"], unit["hkv"], unit["d"], 2)
        what = f"sequences of ctx {unit['ctx']} with {unit['hq']}/{unit['hkv']}/{unit['d']} heads"
    else:
        unit = dict(rows=64, hidden=spec["hidden"], dtype=dtype)
        unit_bytes = 4 * 64 * spec["hidden"] * 2 + spec["hidden"] * 2
        what = f"blocks of 64 rows x {spec['hidden']}"
    with CpuOracleRunner(kind, unit) as runner:
        for _ in range(warmup):
            runner.step()
        times = []
        while sum(times) < seconds or len(times) < 2:
            times.append(runner.step())
        workers = runner.workers
    units = workers * len(times)
    total = sum(times)
    return {
        "value": units * unit_bytes / total / 1e9,
        "unit": "GB/s",
        "cores": workers,
        "kind": "port",
        "sample": f"{units} {what} ({workers} processes x {len(times)} steps, {total:.1f} s), NumPy oracle",
        "seconds_per_step": total / len(times),
        "units_per_step": workers,
        "unit_bytes": unit_bytes,
    }


def run_reference(args, spec: dict) -> None:
    """Reference arm: kernel-lab's CPU path (its NumPy restatement) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    metric = RAGGED_METRIC if spec["kind"] == "ragged" else METRIC
    spec = cpu_unit_spec(spec)
    kind = spec["kind"]
    from oracle.timing import CpuOracleRunner

    if kind == "decode":
        unit = dict(ctx=spec["ctx"], hq=spec["hq"], hkv=spec["hkv"], d=spec["d"], page=spec["page"], dtype="bf16")
        from oracle.oracle import decode_bytes

        unit_bytes = decode_bytes([spec["ctx"]], spec["hq"], spec["hkv"], spec["d"], 2)
    else:
        unit = dict(rows=64, hidden=spec["hidden"], dtype="bf16")
        unit_bytes = 4 * 64 * spec["hidden"] * 2 + spec["hidden"] * 2
    with CpuOracleRunner(kind, unit) as runner:
        for _ in range(args.warmup):
            runner.step()
        times = [runner.step() for _ in range(args.steps)]
        workers = runner.workers
    total = sum(times)
    value = workers * len(times) * unit_bytes / total / 1e9
    line = {
        "metric": metric if kind == "decode" else RMS_METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total / len(times) * 1e3,
        "higher_is_better": True,
        "scaling": spec["scaling"],
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), bf16-rounded)",
        "impl": "reference",
        "config": {"workload": spec["desc"], "sample_per_step": f"{workers} units of the workload"},
        "cpu_baseline": {
            "value": value,
            "unit": "GB/s",
            "cores": workers,
            "kind": "port",
            "sample": f"each step: {workers} sequences/blocks of the workload, one per process",
        },
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU side


def load_traffic(key: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    try:
        return json.loads((REPO / "profiles" / "traffic.json").read_text())[key]["bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


def time_back_to_back(fn, steps: int, stream, launched=None) -> float:
    """Milliseconds per call of `steps` back-to-back calls, CUDA events on the launching stream
    (`launched`, if given, is called once every call is enqueued)."""
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(stream)
    for i in range(steps):
        fn(i)
    b.record(stream)
    if launched is not None:
        launched()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def decode_grid(dev, stream, steps: int, peak: float) -> dict:
    """Config 3's grid (batch {1, 8, 64} x context {512, 4096}, 32/8/128 heads, bf16) on one GPU.
    A cell smaller than L2 rotates over R disjoint replicas of itself (other sequences, other
    pages) whose KV totals more than twice L2, so no launch finds its pages in L2."""
    import torch

    from kernel_lab.kv_cache import random_paged_pool
    from kernel_lab.roofline import decode_attention_work

    op = torch.ops.kernel_lab.paged_decode_attention
    cells = {}
    for B in (1, 8, 64):
        for ctx in (512, 4096):
            w = decode_attention_work([ctx] * B, 32, 8, 128, 2, 2)
            R = max(1, math.ceil(2 * L2_BYTES / w.bytes))
            q, kv = random_paged_pool([ctx] * (B * R), 32, 8, 128, 16, dtype=torch.bfloat16, device=dev,
                                      seed=100 + B + ctx)
            reps = [(q[r * B:(r + 1) * B], kv.block_table[r * B:(r + 1) * B], kv.seq_lens[r * B:(r + 1) * B],
                     torch.empty_like(q[:B])) for r in range(R)]
            scale = 128**-0.5

            def call(i, reps=reps, kv=kv, scale=scale):
                qq, bt, ln, out = reps[i % len(reps)]
                op(out, qq, kv.k_cache, kv.v_cache, bt, ln, scale)

            for i in range(max(3, R)):
                call(i)
            n = max(steps, R)
            ms = time_back_to_back(call, n, stream)
            gbs = w.bytes / (ms * 1e-3) / 1e9
            cells[f"b{B}_ctx{ctx}"] = {"us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                                       "algorithmic_bytes": int(w.bytes), "replicas": R}
            del q, kv, reps
            torch.cuda.empty_cache()
    return cells


def rmsnorm_secondary(dev, stream, steps: int, peak: float) -> dict:
    """Fused add + RMSNorm at 4096 x 8192 bf16 (x, residual ~ N(0,1), weight ~ N(1, 0.1), eps 1e-5),
    back-to-back launches; x, residual and out total 192 MB, more than L2."""
    import torch

    from kernel_lab.roofline import rms_norm_work

    R, H = 4096, 8192
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    res = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    out = torch.empty_like(x)
    op = torch.ops.kernel_lab.fused_add_rms_norm
    for _ in range(3):
        op(out, x, res, w, 1e-5)
    ms = time_back_to_back(lambda i: op(out, x, res, w, 1e-5), max(steps, 20), stream)
    work = rms_norm_work(R, H, 2, True)
    gbs = work.bytes / (ms * 1e-3) / 1e9
    return {"metric": RMS_METRIC, "us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
            "algorithmic_bytes": int(work.bytes), "kernel": "rmsnorm_row_regs", "timing": "back-to-back launches"}


class DecodeE2E:
    """End to end through the public API, the way a serving loop runs: two device slots; step i's
    q, block table and lengths go up from pinned host memory on a copy-in stream and its whole
    output comes back on a copy-out stream, so copies overlap the neighbouring steps' kernels. The
    KV cache stays resident. `decode(q, bt, ln, out_slot)` returns the output tensor to copy out."""

    def __init__(self, decode, q, bt, ln, out_shape, dev, stream):
        import torch

        self.torch = torch
        self.decode = decode
        self.stream = stream
        self.q_h = q.cpu().pin_memory()
        self.bt_h = bt.cpu().pin_memory()
        self.ln_h = ln.cpu().pin_memory()
        self.out_hs = [torch.empty(out_shape, dtype=q.dtype).pin_memory() for _ in range(2)]
        self.slots = [dict(q=torch.empty_like(q), bt=torch.empty_like(bt), ln=torch.empty_like(ln),
                           out=torch.empty_like(q), inputs_free=None, out_read=None) for _ in range(2)]
        self.s_in, self.s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        self.h2d = self.q_h.numel() * self.q_h.element_size() + self.bt_h.numel() * 4 + self.ln_h.numel() * 4
        self.d2h = self.out_hs[0].numel() * self.out_hs[0].element_size()
        self.count = 0

    def step(self):
        torch = self.torch
        i = self.count
        self.count += 1
        sl = self.slots[i % 2]
        with torch.cuda.stream(self.s_in):
            if sl["inputs_free"] is not None:
                self.s_in.wait_event(sl["inputs_free"])  # the kernel two steps back is done with them
            sl["q"].copy_(self.q_h, non_blocking=True)
            sl["bt"].copy_(self.bt_h, non_blocking=True)
            sl["ln"].copy_(self.ln_h, non_blocking=True)
            arrived = torch.cuda.Event()
            arrived.record(self.s_in)
        self.stream.wait_event(arrived)
        if sl["out_read"] is not None:
            self.stream.wait_event(sl["out_read"])  # the copy-out two steps back has read its output
        src = self.decode(sl["q"], sl["bt"], sl["ln"], sl["out"])
        done = torch.cuda.Event()
        done.record(self.stream)
        sl["inputs_free"] = done
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(done)
            self.out_hs[i % 2].copy_(src, non_blocking=True)
            read = torch.cuda.Event()
            read.record(self.s_out)
        sl["out_read"] = read

    def join(self):
        for sl in self.slots:
            if sl["out_read"] is not None:
                self.stream.wait_event(sl["out_read"])

    def run(self, steps: int) -> float:
        """Milliseconds per step over `steps` pipelined steps (after 3 untimed ones)."""
        torch = self.torch
        for _ in range(3):
            self.step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        self.s_in.wait_event(e0)  # no copy of the timed steps starts before the region does
        for _ in range(steps):
            self.step()
        self.join()
        e1.record(self.stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    def last_output(self):
        return self.out_hs[(self.count - 1) % 2]


def main() -> None:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    spec = workload_spec(args.workload, world)
    if args.batch and spec["kind"] in ("decode", "ragged"):
        spec["batch"] = args.batch * (world if spec["scaling"] == "weak" and spec["kind"] == "decode" else 1)
        spec["desc"] += f" (batch overridden: {args.batch})"
    if args.ctx and spec["kind"] == "decode":
        spec["ctx"] = args.ctx
        spec["desc"] += f" (ctx overridden: {args.ctx})"
    if args.heads and spec["kind"] == "decode":
        if world > 1 and spec["layout"] == "kv_heads":
            raise SystemExit("--heads sets one GPU's heads; the KV-head split at N>1 derives them")
        spec["hq"], spec["hkv"] = (int(x) for x in args.heads.split("/"))
        spec["desc"] += f" (heads overridden: {args.heads})"
    if args.batch and spec["kind"] == "rmsnorm":
        spec["rows"] = args.batch
        spec["desc"] += f" (rows overridden: {args.batch})"
    if args.impl == "reference":
        run_reference(args, spec)
        return
    if spec["kind"] == "ragged" and world > 1:
        raise SystemExit("the ragged workload runs on one GPU")

    import torch
    import torch.distributed as dist

    from kernel_lab import cuda_ops
    from kernel_lab.roofline import B200_SPEC_HBM_GBPS, Work, decode_attention_work, measured_peaks, rms_norm_work

    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    if not cuda_ops.available():
        raise SystemExit(f"kernel_lab CUDA path unavailable: {cuda_ops.why_unavailable()}")
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    if world == 1 or rank == 0:
        ClockSampler.init(torch.cuda.current_device())
    peaks = measured_peaks()
    steps = args.steps
    warmup = max(args.warmup, 3)
    gather = None
    extra = {}

    if spec["kind"] == "decode":
        from kernel_lab.kv_cache import random_paged_pool
        from kernel_lab.sharding import PeerHeadGather, batch_range, kv_head_range

        B, ctx, hq, hkv, d, page = (spec[k] for k in ("batch", "ctx", "hq", "hkv", "d", "page"))
        scale = d**-0.5
        if spec["layout"] == "kv_heads":
            lo, hi = kv_head_range(hkv, world, rank)
            b_local = B
            q, kv = random_paged_pool([ctx] * B, hq, hkv, d, page, dtype=torch.bfloat16, device=dev, seed=1234,
                                      kv_head_slice=(lo, hi))
        elif spec.get("cascade"):
            from kernel_lab.kv_cache import PagedKV, random_cascade_problem

            b_lo, b_hi = batch_range(B, world, rank)
            b_local = b_hi - b_lo
            q, ckv = random_cascade_problem([b_local], [spec["prefix"]], [ctx] * b_local, hq, hkv, d, page,
                                            dtype=torch.bfloat16, device=dev, seed=1234 + rank)
            kv = PagedKV(k_cache=ckv.k_cache, v_cache=ckv.v_cache, block_table=ckv.block_table,
                         seq_lens=ckv.seq_lens, page_size=page)
        else:
            b_lo, b_hi = batch_range(B, world, rank)
            b_local = b_hi - b_lo
            q, kv = random_paged_pool([ctx] * b_local, hq, hkv, d, page, dtype=torch.bfloat16, device=dev,
                                      seed=1234 + rank)
        hq_l, hkv_l = q.shape[1], kv.k_cache.shape[2]
        kv_bytes = 1 if spec.get("kv8") else 2
        kernel_work = decode_attention_work([ctx] * b_local, hq_l, hkv_l, d, 2, kv_bytes)  # per rank, per launch
        job_bytes = decode_attention_work([ctx] * B, hq, hkv, d, 2, kv_bytes).bytes
        if spec.get("cascade"):
            # Unique KV bytes: each GPU's shared prefix once plus every sequence's own tokens.
            prefix_kv = spec["prefix"] * hkv * d * 2 * 2
            kernel_work = Work(kernel_work.bytes + prefix_kv,
                               kernel_work.flops + 4 * spec["prefix"] * b_local * hq * d)
            job_bytes += prefix_kv * world
        if spec["layout"] == "kv_heads" and world > 1:
            # The product path at N > 1: one launch per step decodes this rank's KV heads and stores
            # its heads into every rank's output over NVLink.
            gather = PeerHeadGather(B, hq_l, d, torch.bfloat16)

            def decode_op(out_t, q_t, bt_t, ln_t):
                return gather(q_t, kv.k_cache, kv.v_cache, bt_t, ln_t, scale)
        elif spec.get("cascade"):

            def decode_op(out_t, q_t, bt_t, ln_t):
                torch.ops.kernel_lab.paged_decode_attention_cascade(
                    out_t, q_t, kv.k_cache, kv.v_cache, ckv.prefix_block_table, ckv.prefix_lens, ckv.prefix_indptr,
                    bt_t, ln_t, scale, None, None)
                return out_t
        elif spec.get("kv8"):
            from kernel_lab.kv_cache import e4m3_scales, quantize_e4m3

            k_scale, v_scale = e4m3_scales(kv.k_cache), e4m3_scales(kv.v_cache)
            k8, v8 = quantize_e4m3(kv.k_cache, k_scale), quantize_e4m3(kv.v_cache, v_scale)
            kv = type(kv)(k8, v8, kv.block_table, kv.seq_lens, kv.page_size)
            torch.cuda.empty_cache()

            def decode_op(out_t, q_t, bt_t, ln_t):
                torch.ops.kernel_lab.paged_decode_attention_fp8(out_t, q_t, kv.k_cache, kv.v_cache, k_scale, v_scale,
                                                                bt_t, ln_t, scale)
                return out_t
        else:

            def decode_op(out_t, q_t, bt_t, ln_t):
                torch.ops.kernel_lab.paged_decode_attention(out_t, q_t, kv.k_cache, kv.v_cache, bt_t, ln_t, scale)
                return out_t

        out_local = torch.empty_like(q)
        result = [None]

        def step(i=0):
            result[0] = decode_op(out_local, q, kv.block_table, kv.seq_lens)

        metric = FP8_METRIC if spec.get("kv8") else CASCADE_METRIC if spec.get("cascade") else METRIC
        launches_per_step = 3 if spec.get("cascade") else 1
        problems = [(q, kv.block_table, kv.seq_lens, decode_op,
                     (B, hq, d) if gather is not None else tuple(q.shape), job_bytes)]
    elif spec["kind"] == "ragged":
        from kernel_lab.kv_cache import random_paged_pool

        lens = ragged_lens(spec["batch"])
        layouts = {}
        for name, (hq, hkv) in RAGGED_LAYOUTS.items():
            layouts[name] = dict(hq=hq, hkv=hkv, work=decode_attention_work(lens, hq, hkv, 128, 2, 2))
        kernel_work = Work(sum(v["work"].bytes for v in layouts.values()), sum(v["work"].flops for v in layouts.values()))
        job_bytes = kernel_work.bytes
        metric = RAGGED_METRIC
        launches_per_step = 3
    else:
        R, H = spec["rows"], spec["hidden"]
        g = torch.Generator(device=dev).manual_seed(7)
        x = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
        res = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
        out = torch.empty_like(x)
        kernel_work = rms_norm_work(R, H, 2, True)
        job_bytes = kernel_work.bytes * world

        def step(i=0):
            torch.ops.kernel_lab.fused_add_rms_norm(out, x, res, w, 1e-5)

        metric = RMS_METRIC
        launches_per_step = 1

    if spec["kind"] == "ragged":
        # Each layout's pool is built, timed over the same K steps and freed in turn (MHA alone holds
        # 37 GB of KV); a step of the workload is one call per layout, so its time is their sum.
        step_ms = 0.0
        clock_samples = []
        e2e_ms = 0.0
        h2d = d2h = 0
        for name, lay in layouts.items():
            q, kv = random_paged_pool(lens, lay["hq"], lay["hkv"], 128, 16, dtype=torch.bfloat16, device=dev, seed=4)
            out_l = torch.empty_like(q)

            def one(i=0, q=q, kv=kv, out_l=out_l):
                torch.ops.kernel_lab.paged_decode_attention(out_l, q, kv.k_cache, kv.v_cache, kv.block_table,
                                                            kv.seq_lens, 128**-0.5)

            for _ in range(warmup):
                one()
            with ClockSampler(torch.cuda.current_device()) as clocks:
                ms = time_back_to_back(one, steps, stream, clocks.launched)
            clock_samples.append(clocks)
            step_ms += ms
            gbs = lay["work"].bytes / (ms * 1e-3) / 1e9
            lay.update(us=round(ms * 1e3, 2), gbs=round(gbs, 1), frac=round(gbs / peaks.hbm_gbps, 4),
                       algorithmic_bytes=int(lay["work"].bytes), traffic=load_traffic(f"decode_ragged_{name}_n1"),
                       status=cuda_ops.decode_status(clear=True))

            def dec(q_t, bt_t, ln_t, out_t, kv=kv):
                torch.ops.kernel_lab.paged_decode_attention(out_t, q_t, kv.k_cache, kv.v_cache, bt_t, ln_t, 128**-0.5)
                return out_t

            e2e = DecodeE2E(dec, q, kv.block_table, kv.seq_lens, tuple(q.shape), dev, stream)
            lay_e2e = e2e.run(max(10, min(steps, 50)))
            resident = out_l.cpu()
            if not torch.equal(e2e.last_output(), resident):
                raise SystemExit(f"ragged {name}: e2e output differs from the device-resident step's output")
            e2e_ms += lay_e2e
            h2d += e2e.h2d
            d2h += e2e.d2h
            lay["e2e_us"] = round(lay_e2e * 1e3, 2)
            del lay["work"], q, kv, out_l, e2e
            torch.cuda.empty_cache()
        kern_ms = step_ms
        summaries = [c.summary() for c in clock_samples if c.summary()]
        clocks_summary = None
        if summaries:
            clocks_summary = {"sm_mhz": statistics.median(c["sm_mhz"] for c in summaries),
                              "sm_max_mhz": summaries[0]["sm_max_mhz"],
                              "reasons": sorted({r for c in summaries for r in c["reasons"]}),
                              "samples": sum(c["samples"] for c in summaries)}
        extra["layouts"] = layouts
        e2e_line = {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms}
        status = sum(v["status"] for v in layouts.values())
    else:
        for i in range(warmup):
            step(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

        # ---- timed region: exactly K steps, CUDA events on the launching stream. Every step is
        # one launch of the hot path (the fused gather included at N > 1; the cascade's three
        # kernels excepted), so the region's two events give the kernel's average launch duration
        # (an event between back-to-back launches would add ~5 us of launch gap to every step).
        # At N = 1 the clocks are polled inside the timed region. At N > 1 a poll stalls the
        # polled GPU for milliseconds and every rank waits for it at the step's end (2 GPUs: 174 us
        # per step unpolled, 187-204 us with two polls in the region), so the timed region runs
        # unpolled and the same K steps run again straight after it, on every rank, with rank 0
        # polling: the clock record of that repeat stands beside the number, with its own time.
        def timed_steps(sampler_on: bool):
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(torch.cuda.current_device(), period=0.005 if world == 1 else 0.02,
                              enabled=sampler_on and rank == 0) as sampler:
                torch.cuda.synchronize()
                t0.record(stream)
                for i in range(steps):
                    step(i)
                t1.record(stream)
                sampler.launched()
                torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            ms = torch.tensor([t0.elapsed_time(t1) / steps], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            return ms.item(), sampler

        step_ms, clocks = timed_steps(world == 1)
        kern_ms = step_ms
        clocks_summary = clocks.summary()
        if world > 1:
            repeat_ms, clocks = timed_steps(True)
            clocks_summary = clocks.summary()
            if clocks_summary is not None:
                clocks_summary.update(window="the same K steps repeated right after the timed region",
                                      repeat_us_per_step=round(repeat_ms * 1e3, 2))

        # ---- end to end through the public API: pinned host inputs in, result out, every step
        if spec["kind"] == "decode":
            resident = result[0].cpu()  # the timed steps' output, before the e2e steps reuse regions
            q0, bt0, ln0, dec_op, out_shape, _ = problems[0]
            e2e = DecodeE2E(lambda q_t, bt_t, ln_t, out_t: dec_op(out_t, q_t, bt_t, ln_t), q0, bt0, ln0, out_shape,
                            dev, stream)
            if world > 1:
                dist.barrier()
            e2e_ms_local = e2e.run(max(10, min(steps, 100)))
            # The pipelined steps computed what the resident steps did (same inputs, deterministic
            # kernel): a copy that raced its slot would show here.
            if not torch.equal(e2e.last_output(), resident):
                raise SystemExit("e2e output differs from the device-resident step's output")
            h2d, d2h = e2e.h2d, e2e.d2h
        else:
            x_h = x.cpu().pin_memory()
            res_h = res.cpu().pin_memory()
            out_h = torch.empty_like(x_h).pin_memory()
            res_back = torch.empty_like(x_h).pin_memory()
            h2d = 2 * x_h.numel() * 2
            d2h = 2 * out_h.numel() * 2

            def e2e_step(i=0):
                x.copy_(x_h, non_blocking=True)
                res.copy_(res_h, non_blocking=True)
                torch.ops.kernel_lab.fused_add_rms_norm(out, x, res, w, 1e-5)
                out_h.copy_(out, non_blocking=True)
                res_back.copy_(res, non_blocking=True)

            for _ in range(3):
                e2e_step()
            if world > 1:
                dist.barrier()
            e2e_ms_local = time_back_to_back(e2e_step, max(10, min(steps, 100)), stream)
        te = torch.tensor([e2e_ms_local], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = te.item()
        e2e_line = {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(h2d * world),
                    "d2h_bytes_per_step": int(d2h * world), "ms_per_step": e2e_ms}
        if spec["kind"] == "decode":
            status = gather.status(clear=True) if gather is not None else cuda_ops.decode_status(clear=True)
        else:
            status = 0
        if gather is not None and not args.no_extras:
            # Where the step's time goes at N > 1: the same shard through the plain op (no gather),
            # and the gathered step timed again without the clock sampler; max over ranks.
            def plain(i=0):
                torch.ops.kernel_lab.paged_decode_attention(out_local, q, kv.k_cache, kv.v_cache, kv.block_table,
                                                            kv.seq_lens, scale)

            for _ in range(3):
                plain()
            diag = torch.tensor([time_back_to_back(plain, steps, stream), 0.0], device=dev, dtype=torch.float64)
            dist.barrier()
            diag[1] = time_back_to_back(step, steps, stream)
            dist.all_reduce(diag, op=dist.ReduceOp.MAX)
            extra["diagnostics"] = {"shard_plain_op_us": round(diag[0].item() * 1e3, 2),
                                    "gathered_step_no_sampler_us": round(diag[1].item() * 1e3, 2),
                                    "note": "max over ranks; the shard's own kernel without the gather, and the "
                                            "timed step repeated without the NVML clock sampler"}
        if spec["kind"] == "decode" and args.workload == "decode" and world == 1 and not args.no_extras:
            extra["grid"] = decode_grid(dev, stream, min(steps, 100), peaks.hbm_gbps)
            extra["secondary"] = rmsnorm_secondary(dev, stream, steps, peaks.hbm_gbps)

    if gather is not None:
        gather.close()

    if rank == 0:
        achieved = kernel_work.bytes / (kern_ms * 1e-3) / 1e9
        key = f"{args.workload}_n{world}"
        traffic = load_traffic(key)
        if spec["kind"] == "ragged":  # one launch of each layout per step
            per_layout = [v.get("traffic") for v in extra["layouts"].values()]
            traffic = sum(per_layout) if all(t is not None for t in per_layout) else None
        value = job_bytes / (step_ms * 1e-3) / 1e9
        cpu = None
        # kernel-lab has no e4m3 or cascade path to time on the host
        if world == 1 and not args.no_cpu_baseline and not spec.get("kv8") and not spec.get("cascade"):
            cpu = cpu_measure("decode" if spec["kind"] == "ragged" else spec["kind"], spec, args.cpu_seconds)
        layout = spec.get("layout")
        parallelism = ("1 gpu" if world == 1 else f"kv-head tp{world}" if layout == "kv_heads"
                       else f"sequences dp{world}")
        cfg = {"workload": spec["desc"], "l2": L2_NOTE, "parallelism": parallelism}
        if spec["kind"] == "decode":
            cfg.update(batch=spec["batch"], ctx=spec["ctx"], num_q_heads=spec["hq"], num_kv_heads=spec["hkv"],
                       head_dim=spec["d"], page_size=spec["page"], pool_pages=int(kv.k_cache.shape[0]),
                       algorithmic_bytes_per_gpu=int(kernel_work.bytes), planner="load-balanced (num_splits=0)")
            if gather is not None:
                cfg["gather"] = ("fused: the decode kernel stores every rank's heads into every rank's output over "
                                 "NVLink (CUDA IPC peer stores, no multicast), one launch per step")
        elif spec["kind"] == "ragged":
            cfg.update(batch=spec["batch"], head_dim=128, page_size=16, lengths="U[1, 32768] seed 4 + 16383/16384/16385",
                       layouts={k: f"{hq}/{hkv}" for k, (hq, hkv) in RAGGED_LAYOUTS.items()})
        else:
            cfg.update(rows=spec["rows"], hidden=spec["hidden"], eps=1e-5)
        if "grid" in extra:
            cfg["grid_l2"] = "cells smaller than 2x L2 rotate over disjoint replicas totalling more than 2x L2"
        kernel_name = ("cascade_prefix_kernel + cascade_prefix_reduce_kernel + decode_tc_kernel (the whole op)"
                       if spec.get("cascade") else "decode_tc_kernel (attention and head gather in one launch)"
                       if gather is not None else "decode_tc_kernel" if spec["kind"] in ("decode", "ragged")
                       else "rmsnorm_row_regs")
        line = {
            "metric": metric,
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": step_ms,
            "us_per_call": kern_ms * 1e3,
            "pct_of_spec_peak_hbm": 100 * achieved / B200_SPEC_HBM_GBPS,
            "higher_is_better": True,
            "scaling": spec["scaling"],
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/K/V, shuffled pages, NaN spare pages)" if spec["kind"] != "rmsnorm"
            else "synthetic (seeded x, residual ~ N(0,1), weight ~ N(1, 0.1))",
            "impl": "b200",
            "config": cfg,
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peaks.hbm_gbps,
                "unit": "GB/s",
                "frac": achieved / peaks.hbm_gbps,
                "peak_source": f"{peaks.source} (MEASURED_PEAKS.json hbm_gbs, copy burst)"
                if peaks.source == "measured" else "fallback 6650 GB/s",
                "traffic": traffic,
                "algorithmic_bytes_per_launch": int(kernel_work.bytes) if spec["kind"] != "ragged"
                else "per layout, see layouts",
                "kernel": kernel_name,
            },
            "cpu_baseline": cpu,
            "e2e": e2e_line,
            "clocks": clocks_summary,
            "gpu_launches": steps * launches_per_step,
            "status_bits": status,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
