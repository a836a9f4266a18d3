#!/usr/bin/env python3
"""Benchmark of the emmy B200 backend on BASELINE.json's configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c3|c4|c5]

One JSON line on stdout (rank 0).  A "step" is one pass of the hot path over
one batch: one launch of the KernelOp compiled from the config's IR, on
inputs already resident in HBM (``value``), and the same call through the
C ABI on pinned host buffers with the copies inside the timed region
(``e2e``).  The default workload is BASELINE configs[1] (the metric's
HBM-bound pointwise chain, y = GELU_tanh(x*s + t) on f32 [16384, 16384]).
Under torchrun every rank runs its own full-size shard (weak scaling, no
data-path collective) and the slowest rank's device time is reported.

``--impl reference`` times the reference's CPU restatement (oracle/) on
the host cores, for the same metric, on a bounded sample per step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

REPO = Path(__file__).resolve().parent
CASES = REPO / "tests" / "golden" / "cases"
METRIC = "HBM GB/s (pointwise/reduce), GEMM TFLOP/s; % of B200 roofline at 1/2/4/8 GPU"
sys.path.insert(0, str(REPO))

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the
# dominant kernel, from single-launch ncu captures (cold L2) of the same
# kernels; the captures and commands are summarised in
# profiles/dram_traffic_per_launch.md.  c4 is the 2^28-element capture scaled
# by 8 (a streaming sum's traffic grows with its input).
DRAM_TRAFFIC = {
    "c2_gelu_full": 1073930240 + 1024718592,
    "c3_rowsummax_full": 2147724544 + 3113472,
    "c4_sum_full": 8 * (1073763072 + 3136256),
    "c5_gemm_full": 6476781312 + 532221952,
}

CONFIGS = {
    # name: (case dir, unit, bound, algorithmic units per launch, workload text)
    # C1 is launch-latency bound: its line reports microseconds per launch (lower is better)
    "c1": ("c1_add_64", "us", "latency", 3 * 64 * 4,
           "BASELINE configs[0]: c = a + b, f32 [64], one 256-thread block (launch latency)"),
    "c2": ("c2_gelu_full", "GB/s", "hbm", 2 * (1 << 28) * 4 + 2 * 16384 * 4,
           "BASELINE configs[1]: y = GELU_tanh(x*s + t), x f32 [16384, 16384], s,t f32 [16384]"),
    "c3": ("c3_rowsummax_full", "GB/s", "hbm", (1 << 31) + 2 * 8192 * 4,
           "BASELINE configs[2]: row sum and max of f32 [8192, 65536]"),
    "c4": ("c4_sum_full", "GB/s", "hbm", (1 << 33) + 4,
           "BASELINE configs[3]: sum of f32 [2^31]"),
    "c5": ("c5_gemm_full", "TFLOP/s", "tensor", 2 * 16384 * 16384 * 8192,
           "BASELINE configs[4]: relu(A@B + bias), A bf16 [16384, 8192], B bf16 [8192, 16384]"),
    # fused row reduction + pointwise (the next row of the scope table, not a BASELINE config):
    # algorithmic bytes = one read of x, one write of y (+ the weight vector)
    "f_rmsnorm": ("f_rmsnorm_bench_16384x8192", "GB/s", "hbm", 2 * 16384 * 8192 * 4 + 8192 * 4,
                  "row-fused rmsnorm: y = x * rsqrt(mean(x^2) + 1e-6) * w, x f32 [16384, 8192]"),
    "f_softmax": ("f_softmax_bench_16384x8192", "GB/s", "hbm", 2 * 16384 * 8192 * 4,
                  "row-fused softmax over rows of x f32 [16384, 8192]"),
    "f_l2norm": ("f_l2norm_bench_16384x8192", "GB/s", "hbm", 2 * 16384 * 8192 * 4,
                 "row-fused l2norm: y = x * rsqrt(sum(x^2) + 1e-12), x f32 [16384, 8192]"),
    # naive-attention IR, f32 on CUDA cores (exact reference arithmetic): algorithmic FLOP =
    # q.k^T and p.v once each, 2 * 2 * seq^2 * dim
    "a_attn": ("a_attn_bench_2048x64", "TFLOP/s", "fp32", 4 * 2048 * 2048 * 64,
               "naive attention softmax(q k^T / sqrt(64)) v, q,k,v f32 [2048, 64]"),
}
# nominal FP32 CUDA-core peak: 148 SMs x 128 lanes x 2 FLOP x 1.965 GHz
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
L2_BYTES = 126 * 1024 * 1024
L2_FLUSH_BYTES = 256 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return json.loads(p.read_text()), "measured"
        except json.JSONDecodeError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of the job's GPUs, sampled
    through NVML (read-only queries) while the timed region runs.

    One sampler per job, on rank 0, polls every GPU of the node the job uses
    (devices 0..world-1 of this process's view) every ~3 ms.  NVML is opened
    before the timed region; ``start``/``stop`` only run the polling thread,
    so the timed region pays no NVML set-up.  With one poller per rank,
    eight ranks' NVML calls slowed the host's launch loop enough to stretch
    steps that end in a collective."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}
    INTERVAL_S = 0.003

    def __init__(self, devices: list[int], active: bool = True):
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handles = []
        if not active:
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handles = [pynvml.nvmlDeviceGetHandleByIndex(self._physical_index(d)) for d in devices]
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handles[0], pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    @staticmethod
    def _physical_index(device: int) -> int:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            try:
                return int(vis.split(",")[device])
            except (ValueError, IndexError):
                pass
        return device

    def start(self) -> None:
        if self._nvml is None:
            return
        pynvml = self._nvml

        def run():
            while not self._stop.is_set():
                for h in self._handles:
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, rs))
                    except pynvml.NVMLError:
                        pass
                self._stop.wait(self.INTERVAL_S)
        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def close(self) -> None:
        self.stop()
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass
            self._nvml = None

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml unavailable" if self._nvml is None and not self._handles else "nvml, no sample"}
        reasons = sorted(name for name, bit in self.REASONS.items()
                         if any(rs & bit for _, rs in self.samples))
        return {"sm_mhz": statistics.median(sm for sm, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "gpus": len(self._handles),
                "source": f"nvml from rank 0, every {self.INTERVAL_S * 1e3:.0f} ms, all GPUs of the job"}


# ---------------------------------------------------------------------------- inputs


def make_inputs(cfg: str, spec, rank: int, device: str):
    """Seeded synthetic inputs with the config's shapes and distributions
    (generated on the device; per-rank seeds for weak scaling)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(1234 + 7919 * rank)
    out = {}
    for name in spec.arg_order:
        a = spec.args[name]
        shape = tuple(a["shape"]) or (1,)
        dt = {"f32": torch.float32, "bf16": torch.bfloat16}[a.get("dtype", "f32")]
        if a.get("output"):
            out[name] = torch.empty(shape, dtype=dt, device=device)
            continue
        init = a.get("init", {"kind": "normal", "std": 1.0, "mean": 0.0})
        if init["kind"] == "uniform":
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.uniform_(init["low"], init["high"], generator=g)
        else:
            t = torch.randn(shape, dtype=torch.float32, device=device, generator=g)
            t.mul_(init.get("std", 1.0)).add_(init.get("mean", 0.0))
        out[name] = t.to(dt)
    return out


# ---------------------------------------------------------------------------- distributed glue


def max_over_ranks(value: float, world: int, device) -> float:
    """The slowest rank's time (every rank must call this, in the same order)."""
    if world <= 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def combine_step(cfg: str, bufs: dict, world: int):
    """The path's one exchange: a full-array sum over N GPUs adds the per-GPU
    partial sums (NCCL all-reduce of one float, enqueued on the current
    stream).  Every other config shards with no collective."""
    if cfg != "c4" or world <= 1:
        return lambda: None
    import torch
    out = bufs["sum_1"]
    return lambda: torch.distributed.all_reduce(out, op=torch.distributed.ReduceOp.SUM)


# ---------------------------------------------------------------------------- our arm


def run_ours(args, rank: int, world: int, local: int) -> dict | None:
    import torch
    from emmy_ptx_compiler_b200 import compiler, harness, runtime

    device = f"cuda:{local}"
    torch.cuda.set_device(local)
    case_id, unit, bound, units, workload = CONFIGS[args.config]
    spec = harness.load_case(CASES / case_id)
    bundle = compiler.compile_bundle(spec.ir_path, want_cubin=True)
    runtime.init(local)
    mod = runtime.Module(bundle["cubin"], spec.entry, local)
    # the geometry actually launched (pointwise grids are sized by the loader from occupancy)
    launch = {"grid": list(mod.grid), "block": list(mod.block), "smem": mod.smem}
    bufs = make_inputs(args.config, spec, rank, device)
    order = [bufs[n] for n in spec.arg_order]
    stream = torch.cuda.current_stream(local).cuda_stream

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    combine = combine_step(args.config, bufs, world)
    go = mod.bind(order, stream=stream)  # argument words prepared once: one C-ABI call per launch
    step = go if args.config != "c4" or world <= 1 else (lambda: (go(), combine()))
    xchg = None
    if args.config == "c4" and world > 1 and args.combine == "fused":
        # one kernel per GPU: shard sum fused with the combine over NVLink peer memory
        xchg = runtime.Exchange(local, world, rank)
        handles = [None] * world
        torch.distributed.all_gather_object(handles, xchg.handle)
        xchg.connect(handles)
        x_in, total, n_in = bufs["x"], bufs["sum_1"], bufs["x"].numel()
        step = lambda: xchg.sum_allreduce(x_in, n_in, total, timeout_ms=10000, stream=stream)  # noqa: E731

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(local)
    st = mod.status()
    if st:
        raise RuntimeError(f"kernel status 0x{st:x} during warm-up")
    clocks = ClockSampler(list(range(min(world, torch.cuda.device_count()))) if world > 1 else [local],
                          active=(rank == 0))
    # inputs smaller than L2 would stay cached across steps: each step then runs
    # after a write of a buffer larger than L2 and is timed by its own events
    footprint = sum(t.numel() * t.element_size() for t in bufs.values())
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device) if footprint < L2_BYTES else None
    barrier()
    torch.cuda.synchronize(local)
    clocks.start()
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize(local)
        timed_ms = e0.elapsed_time(e1)
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for a, b in ev:
            flush.fill_(1)
            a.record()
            step()
            b.record()
        torch.cuda.synchronize(local)
        timed_ms = sum(a.elapsed_time(b) for a, b in ev)
    clocks.stop()
    barrier()
    clocks.close()
    if xchg is not None:
        xst = xchg.status()
        xchg.close()
        if xst:
            raise RuntimeError(f"fused sum + combine status 0x{xst:x} (a peer did not arrive in time)")
    ms_max = max_over_ranks(timed_ms, world, device)
    per_launch_ms = ms_max / args.steps
    latency = unit == "us"
    graph = None
    if latency:
        # back to back: the rate at which the host can submit bound launches
        torch.cuda.synchronize(local)
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        for _ in range(args.steps):
            go()
        b1.record()
        torch.cuda.synchronize(local)
        back_to_back_us = b0.elapsed_time(b1) * 1e3 / args.steps
        # the same launches recorded once as a CUDA graph and replayed: device
        # time per launch without the host's per-launch submission cost
        gs = torch.cuda.Stream(device=local)
        torch.cuda.synchronize(local)
        with runtime.Graph.record(local, gs.cuda_stream) as g:
            for _ in range(args.steps):
                mod.launch(order, stream=gs.cuda_stream)
        for _ in range(args.warmup):
            g.launch(gs.cuda_stream)
        torch.cuda.synchronize(local)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(gs)
        g.launch(gs.cuda_stream)
        g1.record(gs)
        torch.cuda.synchronize(local)
        graph = {"graph_replay_us_per_launch": round(g0.elapsed_time(g1) * 1e3 / args.steps, 3),
                 "launches_per_graph": args.steps, "graph_path": "emmy_graph_begin/end/launch (C ABI)",
                 "back_to_back_us_per_launch": round(back_to_back_us, 3),
                 "note": "value: one launch timed alone after an L2 flush; the back-to-back and graph "
                         "figures run with L2 warm"}
        g.close()
    if latency:
        value = achieved = per_launch_ms * 1e3
    else:
        value = units * world * args.steps / (ms_max / 1e3) / (1e9 if unit == "GB/s" else 1e12)
        achieved = units / (per_launch_ms / 1e3) / (1e9 if unit == "GB/s" else 1e12)
    pk, pk_kind = peaks()
    peak = pk["hbm_gbs"] if bound == "hbm" else pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    if bound == "fp32":
        peak, pk_kind = round(FP32_NOMINAL_TFLOPS, 1), "nominal"
    peak_key = {"hbm": "hbm_gbs", "tensor": "bf16_tflops", "fp32": "fp32 CUDA cores", "latency": "none"}[bound]
    traffic = DRAM_TRAFFIC.get(case_id)

    # e2e: the C-ABI host-buffer call, copies in the timed region
    host = {}
    nbytes, roles, ptrs = [], [], []
    for name in spec.arg_order:
        t = bufs[name]
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        if not spec.args[name].get("output"):
            h.copy_(t)
        host[name] = h
        ptrs.append(h.data_ptr())
        nbytes.append(h.numel() * h.element_size())
        roles.append(runtime.EMMY_ROLE_OUT if spec.args[name].get("output") else runtime.EMMY_ROLE_IN)
    e2e_steps = max(1, args.steps if latency else min(args.steps, 5))
    mod.run_host(ptrs, nbytes, roles, stream=stream)  # warm the module's device buffers
    barrier()
    torch.cuda.synchronize(local)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        mod.run_host(ptrs, nbytes, roles, stream=stream)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, device)
    h2d = sum(b for b, r in zip(nbytes, roles) if r == runtime.EMMY_ROLE_IN)
    d2h = sum(b for b, r in zip(nbytes, roles) if r == runtime.EMMY_ROLE_OUT)
    e2e_value = (e2e_s / e2e_steps * 1e6 if latency
                 else units * world * e2e_steps / e2e_s / (1e9 if unit == "GB/s" else 1e12))

    ref_ptx = None
    if rank == 0 and world == 1 and (args.config in ("c1", "c2") or args.config[:2] in ("f_", "a_")) \
            and not args.no_ref_ptx:
        ref_ptx = time_reference_ptx(spec, bufs, local, units, unit)

    mod.close()
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": not latency,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if args.config != "c5" else "bf16",
        "data": "synthetic (seeded on device, BASELINE distributions)",
        "config": {"workload": workload, "case": case_id, "rows_per_rank": spec.args[spec.arg_order[0]]["shape"][0],
                   "parallelism": f"{world} ranks, each its own full-size shard; no collective",
                   "l2": ("inputs larger than L2 (126 MB), no flush needed" if flush is None else
                          f"working set {footprint} B < L2: a {L2_FLUSH_BYTES >> 20} MiB buffer is written before "
                          "every timed step, and each step is timed by its own CUDA events"),
                   "launch": launch},
        "roofline": ({"bound": bound, "achieved": round(achieved, 2), "peak": peak,
                      "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic,
                      "peak_source": f"{pk_kind} ({peak_key})",
                      "units_per_launch": units} if not latency else
                     {"bound": "latency", "achieved": round(achieved, 3), "peak": None, "unit": "us", "frac": None,
                      "traffic": None, "units_per_launch": units,
                      "note": "768 bytes per launch: bounded by launch latency, not by HBM or tensor cores"}),
        "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": "emmy_run_host (C ABI) on pinned host buffers"},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if ref_ptx is not None:
        line["reference_ptx_gpu"] = ref_ptx
    if graph is not None:
        line["latency"] = graph
    if args.config == "c4" and world > 1:
        line["config"]["parallelism"] = (
            f"{world} ranks, each its own 2^31-element shard; every step is one kernel per GPU that sums "
            "the shard and combines the per-GPU totals over NVLink peer memory (emmy_sum_f32_allreduce)"
            if args.combine == "fused" else
            f"{world} ranks, each its own 2^31-element shard; the per-rank sums are combined by an NCCL "
            "all-reduce inside every step")
        line["gpu_launches"] = args.steps
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.config, seconds=args.cpu_seconds)
    return line


def time_reference_ptx(spec, bufs, local: int, units: int, unit: str) -> dict:
    """The reference compiler's own PTX for the same IR on the same B200
    (JIT-loaded, meta.json launch), on the same device buffers."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    ref = spec.root / "ref.ptx"
    if not ref.is_file():
        return {"unavailable": "no reference PTX for this IR"}
    mod = runtime.Module(ref.read_bytes(), spec.entry, local)
    g, b = spec.kernel["grid"], spec.kernel["block"]
    order = [bufs[n] for n in spec.arg_order]
    stream = torch.cuda.current_stream(local).cuda_stream
    for _ in range(3):
        mod.launch(order, stream=stream, grid=g, block=b)
    torch.cuda.synchronize(local)
    n = 50 if unit == "us" else 5
    footprint = sum(t.numel() * t.element_size() for t in bufs.values())
    flush = (torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=f"cuda:{local}")
             if footprint < L2_BYTES else None)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for e0, e1 in ev:    # same rule as our arm: an L2 flush before each launch of a small working set
        if flush is not None:
            flush.fill_(1)
        e0.record()
        mod.launch(order, stream=stream, grid=g, block=b)
        e1.record()
    torch.cuda.synchronize(local)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / n
    mod.close()
    value = ms * 1e3 if unit == "us" else units / (ms / 1e3) / (1e9 if unit == "GB/s" else 1e12)
    return {"value": round(value, 3), "unit": unit,
            "ms_per_launch": round(ms, 4), "launch": {"grid": g, "block": b}}


# ---------------------------------------------------------------------------- CPU arms


# bounded CPU samples of each workload for the oracle arms: (rows per task, text)
CPU_SAMPLES = {
    "c1": (1, "calls of the 64-element add, one thread"),
    "c2": (16, "rows of the GELU chain over 16384 columns"),
    "c3": (4, "rows of 65536 reduced (sum and max) in the reference's strided schedule order"),
    "c4": (1, "a 2^20+3-element full sum in the reference's strided schedule order"),
    "c5": (1, "rows of A (1 x 8192) times B (8192 x 16384), sequential fma over k, plus bias and ReLU"),
    "f_rmsnorm": (16, "rows of 8192 through the row-fused IR in the reference's order (strided sums, tree)"),
    "f_softmax": (16, "rows of 8192 through the row-fused IR in the reference's order (strided sums, tree)"),
    "f_l2norm": (16, "rows of 8192 through the row-fused IR in the reference's order (strided sums, tree)"),
    "a_attn": (64, "query rows of the naive attention IR over all 2048 keys (oracle.c restatement: scores and "
                   "exponentials once per key, sequential fma order)"),
}


def _scaled(kop, axes):
    """``kop`` with its Tile's axes replaced (extents of a bounded sample)."""
    import copy
    from emmy._core import Axis, Dim
    tile = copy.copy(list(kop.body)[0])
    tile.axes = tuple(Axis(n, Dim(e)) for n, e in axes)
    k2 = copy.copy(kop)
    k2.body = (tile,)
    return k2


def _oracle_sample(cfg: str, rows: int):
    """(callable, algorithmic units it processes) for a bounded CPU sample of
    the config's workload, evaluated by the oracle (oracle/interp.py)."""
    import numpy as np
    sys.path.insert(0, str(REPO / "oracle"))
    import interp
    case_id, unit, bound, units, _ = CONFIGS[cfg]
    rng = np.random.default_rng(0)
    if cfg == "c1":
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / case_id)
        ins = {n: rng.standard_normal(tuple(shapes[n])).astype(np.float32) for n in ("a", "b")}
        fn = lambda: interp.evaluate(kop, shapes, dtypes, ins, {"c": tuple(shapes["c"])})  # noqa: E731
        return fn, units
    if cfg == "c2":
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / case_id)
        cols = 16384
        shp = dict(shapes, x=(rows, cols), y=(rows, cols))
        ins = {"x": rng.standard_normal((rows, cols), dtype=np.float32),
               "s": rng.uniform(0.5, 1.5, cols).astype(np.float32),
               "t": rng.uniform(-0.1, 0.1, cols).astype(np.float32)}
        k2 = _scaled(kop, [("a0", rows), ("a1", cols)])
        fn = lambda: interp.evaluate(k2, shp, dtypes, ins, {"y": (rows, cols)})  # noqa: E731
        return fn, rows * cols * 8 + 2 * cols * 4
    if cfg == "c3":
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / case_id)
        cols = 65536
        axes = [(a.name, int(a.extent.value)) for a in list(kop.body)[0].axes]
        shp = dict(shapes, x=(rows, cols), sum_1=(rows,), max_1=(rows,))
        ins = {"x": rng.standard_normal((rows, cols), dtype=np.float32)}
        k2 = _scaled(kop, [(axes[0][0], rows)] + axes[1:])
        fn = lambda: interp.evaluate(k2, shp, dtypes, ins, {"sum_1": (rows,), "max_1": (rows,)})  # noqa: E731
        return fn, rows * cols * 4 + 2 * rows * 4
    if cfg == "c4":
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / "c4_sum_1048579")
        n = int(shapes["x"][0])
        ins = {"x": rng.uniform(-1, 1, n).astype(np.float32)}
        fn = lambda: interp.evaluate(kop, shapes, dtypes, ins, {"sum_1": ()})  # noqa: E731
        return fn, n * 4 + 4
    if cfg == "c5":
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / case_id)
        K, N = 8192, 16384
        shp = dict(shapes, A=(rows, K), C=(rows, N))
        ins = {"A": interp.bf16_round(rng.normal(0, 0.02, (rows, K)).astype(np.float32)),
               "B": interp.bf16_round(rng.normal(0, 0.02, (K, N)).astype(np.float32)),
               "bias": rng.normal(0, 0.02, N).astype(np.float32)}
        k2 = _scaled(kop, [("i", rows), ("j", N)])
        fn = lambda: interp.evaluate(k2, shp, dtypes, ins, {"C": (rows, N)})  # noqa: E731
        return fn, 2 * rows * N * K
    if cfg in ("f_rmsnorm", "f_softmax", "f_l2norm"):
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / case_id)
        cols = int(shapes["x"][1])
        axes = [(a.name, int(a.extent.value)) for a in list(kop.body)[0].axes]
        shp = dict(shapes, x=(rows, cols), y=(rows, cols))
        ins = {"x": rng.standard_normal((rows, cols), dtype=np.float32)}
        if "w" in shapes:
            ins["w"] = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        k2 = _scaled(kop, [(axes[0][0], rows)] + axes[1:])
        fn = lambda: interp.evaluate(k2, shp, dtypes, ins, {"y": (rows, cols)})  # noqa: E731
        return fn, 2 * rows * cols * 4 + (cols * 4 if "w" in shapes else 0)
    if cfg == "a_attn":
        # the C restatement of the naive attention IR (oracle/oracle.c), pinned to
        # the Python oracle and the reference's golden vectors by the CPU tests
        kop, meta, mk, shapes, dtypes = interp.load_case(CASES / case_id)
        seq, dim = shapes["q"]
        q = rng.standard_normal((rows, dim), dtype=np.float32)
        kt = rng.standard_normal((dim, seq), dtype=np.float32)
        v = rng.standard_normal((seq, dim), dtype=np.float32)
        out = np.empty((rows, dim), dtype=np.float32)
        scale = float(np.float32(1.0 / np.sqrt(dim)))
        L = interp.lib()

        def fn():
            o = np.empty_like(out)
            if L.ora_attn_naive_f32(interp._p(q), interp._p(kt), interp._p(v), interp._p(o),
                                    rows, seq, dim, dim, scale) != 0:
                raise MemoryError("oracle scratch")
        return fn, 4 * rows * seq * dim
    raise ValueError(f"no CPU sample defined for {cfg}")


def _units_scale(unit: str) -> float:
    return 1e9 if unit == "GB/s" else 1e12


def cpu_baseline(cfg: str, seconds: float = 10.0) -> dict:
    """The oracle port on the host cores: samples split over a thread pool
    (numpy and the oracle's C loops release the GIL)."""
    if cfg not in CPU_SAMPLES:
        return {"unavailable": f"CPU baseline for {cfg} not wired"}
    unit = CONFIGS[cfg][1]
    threads = len(os.sched_getaffinity(0))
    rows_per_task, what = CPU_SAMPLES[cfg]
    fn, units = _oracle_sample(cfg, rows_per_task)
    fn()  # warm
    if unit == "us":
        calls, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(seconds, 2.0):
            fn()
            calls += 1
        el = time.perf_counter() - t0
        return {"value": round(el / calls * 1e6, 3), "unit": unit, "cores": 1, "kind": "port",
                "sample": f"oracle/interp.py, {calls} {what}"}
    done_units = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        while time.perf_counter() - t0 < seconds:
            list(ex.map(lambda _: fn(), range(threads)))
            done_units += units * threads
    el = time.perf_counter() - t0
    return {"value": round(done_units / el / _units_scale(unit), 4), "unit": unit, "cores": threads, "kind": "port",
            "sample": f"oracle port (oracle/), {threads} threads x {rows_per_task} {what} per round, "
                      f"{el:.1f} s of rounds"}


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    case_id, unit, bound, units, workload = CONFIGS[args.config]
    if args.config not in CPU_SAMPLES:
        return {"impl": "reference", "unavailable": f"reference CPU arm not wired for {args.config}"}
    threads = len(os.sched_getaffinity(0))
    rows_per_task, what = CPU_SAMPLES[args.config]
    fn, units_task = _oracle_sample(args.config, rows_per_task)
    if unit == "us":
        # a latency config: one call at a time on one thread, microseconds per call
        for _ in range(args.warmup):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        el = time.perf_counter() - t0
        us = el / args.steps * 1e6
        return {"metric": METRIC, "value": round(us, 3), "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": False,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": {"workload": workload, "case": case_id},
                "cpu_baseline": {"value": round(us, 3), "unit": unit, "cores": 1, "kind": "port",
                                 "sample": f"{args.steps} {what}"},
                "e2e": {"value": round(us, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    with ThreadPoolExecutor(max_workers=threads) as ex:
        for _ in range(args.warmup):
            list(ex.map(lambda _: fn(), range(threads)))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            list(ex.map(lambda _: fn(), range(threads)))
        el = time.perf_counter() - t0
    value = units_task * threads * args.steps / el / _units_scale(unit)
    return {"metric": METRIC, "value": round(value, 4), "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32" if args.config != "c5" else "bf16",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": workload, "case": case_id},
            "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": "port",
                             "sample": f"{threads} threads x {rows_per_task} {what} per step"},
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main() -> int:
    # stdout carries exactly one JSON line: native libraries (NCCL prints its
    # version banner on fd 1) are pointed at stderr, the line goes to a copy
    # of the original stdout
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    out = os.fdopen(json_fd, "w")
    try:
        return _main(out)
    finally:
        out.flush()


def _main(out) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-ptx", action="store_true")
    ap.add_argument("--combine", choices=["fused", "nccl"], default="nccl",
                    help="c4 at N>1: our reduction kernel + NCCL all-reduce (measured faster), or the fused "
                         "sum + NVLink peer combine kernel")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), file=out, flush=True)
        return 0
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device(f"cuda:{local}"))
    try:
        line = run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()
    if line is not None:
        print(json.dumps(line), file=out, flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
