#!/usr/bin/env python3
"""Benchmark of the emmy B200 backend on BASELINE.json's configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1|c2|c3|c4|c5|f_*|a_attn] [--only]

One JSON line on stdout (rank 0).  A "step" is one pass of the hot path over
one batch: one launch of the KernelOp compiled from the config's IR, on
inputs already resident in HBM (``value``), and the same call through the
C ABI on pinned host buffers with the copies inside the timed region
(``e2e``).  The default workload is BASELINE configs[1] (the metric's
HBM-bound pointwise chain, y = GELU_tanh(x*s + t) on f32 [16384, 16384]);
the same run then times configs[2..4] (C3 row sum+max, C4 full sum, C5
GEMM) the same way and reports them under ``configs``, each with its own
roofline, e2e, reference-PTX and CPU baselines.

Under torchrun (N > 1) the BASELINE problem is split over the ranks
(strong scaling): rows / N per rank for C2, C3 and C5 (B replicated), 2^31 / N
elements for C4 with the per-rank partial sums combined by an NCCL
all-reduce inside every step; each rank compiles the KernelOp for its own
shard (emmy_ptx_compiler_b200.shard) and checks its own result.  A weak
pass (every rank a full-size copy) is reported beside it under ``weak``.
The slowest rank's device time is reported.

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
    "c2_gelu_full": 1073916928 + 1023762432,
    "c3_rowsummax_full": 2147724544 + 3113472,
    "c4_sum_full": 8 * (1073763072 + 3136256),
    "c5_gemm_full": 5619480320 + 530271232,
    # q, k, v read once from DRAM (1.5 MiB); the output stays in L2 within the launch
    "a_attn_bench_2048x64": 1618944 + 256,
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
    # naive-attention IR, f32 operands on the tensor cores (tf32 with a three-term split):
    # algorithmic FLOP = q.k^T and p.v once each, 2 * 2 * seq^2 * dim
    "a_attn": ("a_attn_bench_2048x64", "TFLOP/s", "tf32x3", 4 * 2048 * 2048 * 64,
               "naive attention softmax(q k^T / sqrt(64)) v, q,k,v f32 [2048, 64]"),
}
# nominal FP32 CUDA-core peak: 148 SMs x 128 lanes x 2 FLOP x 1.965 GHz
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# nominal dense tf32 tensor peak; every f32 product of the attention kernel takes three
# tf32 MMAs (hi*hi + hi*lo + lo*hi), so its algorithmic ceiling is a third of it
TF32_NOMINAL_TFLOPS = 1100.0
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


def make_inputs(spec, shapes: dict, rank: int, device: str, row0: dict | None = None):
    """Seeded synthetic inputs with the config's distributions and the shapes
    this rank holds (its shard under strong scaling, generated on the device)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(1234 + 7919 * rank)
    out = {}
    for name in spec.arg_order:
        a = spec.args[name]
        shape = tuple(shapes.get(name, a["shape"])) or (1,)
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
    if CONFIGS[cfg][2] != "hbm" or cfg != "c4" or world <= 1:
        return lambda: None
    import torch
    out = bufs["sum_1"]
    return lambda: torch.distributed.all_reduce(out, op=torch.distributed.ReduceOp.SUM)


# ---------------------------------------------------------------------------- our arm


class Job:
    """One config compiled and resident on this rank: the whole problem
    (N = 1, or weak scaling), or this rank's shard of it (strong scaling,
    emmy_ptx_compiler_b200.shard)."""

    def __init__(self, cfg: str, rank: int, world: int, local: int, mode: str, combine: str = "fused"):
        import torch
        from emmy_ptx_compiler_b200 import compiler, frontend, harness, runtime, shard
        self.cfg, self.rank, self.world, self.local, self.mode = cfg, rank, world, local, mode
        self.device = f"cuda:{local}"
        case_id, self.unit, self.bound, self.units, self.workload = CONFIGS[cfg]
        self.case_id = case_id
        self.spec = harness.load_case(CASES / case_id)
        raw = json.loads(self.spec.ir_path.read_text())
        info = frontend.load_graph(raw)
        args = frontend.arg_order_for(info.kop, self.spec.kernel)
        shapes, dtypes = frontend.load_shapes(raw, info.kop, self.spec.kernel)
        self.shard = None
        if mode == "strong" and world > 1:
            self.shard = shard.shard_kernel(info.kop, shapes, world, rank)
            comp = compiler.Compiler(self.shard.kop, self.shard.shapes, dtypes, args, self.spec.kernel)
            self.shapes = self.shard.shapes
        else:
            comp = compiler.Compiler(info.kop, shapes, dtypes, args, self.spec.kernel)
            self.shapes = shapes
        self.notes = comp.lower().kernel.notes
        runtime.init(local)
        self.mod = runtime.Module(comp.cubin(), self.spec.entry, local)
        self.launch = {"grid": list(self.mod.grid), "block": list(self.mod.block), "smem": self.mod.smem}
        self.bufs = make_inputs(self.spec, self.shapes, rank, self.device)
        self.order = [self.bufs[n] for n in self.spec.arg_order]
        self.stream = torch.cuda.current_stream(local).cuda_stream
        self.go = self.mod.bind(self.order, stream=self.stream)
        # a full-array reduction's per-GPU results are combined in every step
        # (weak scaling too: every rank then sums its own full-size copy)
        self.partial = ((self.shard is not None and self.shard.mode == "partial")
                        or (mode == "weak" and world > 1 and cfg == "c4"))
        if mode == "weak":
            combine = "nccl"
        self.step = self.go
        self.xchg = None
        self.combine = None
        if self.partial and combine == "fused" and self.notes.get("cross_gpu_entry"):
            # one kernel per GPU: the shard's reduction ends with the exchange of the
            # per-GPU results over NVLink peer memory (the module's <entry>__xchg)
            self.xchg = runtime.Exchange(local, world, rank)
            handles = [None] * world
            torch.distributed.all_gather_object(handles, self.xchg.handle)
            self.xchg.connect(handles)
            self.step = self.xchg.bind(self.mod, self.order, timeout_ms=10000, stream=self.stream)
            self.combine = "fused: the KernelOp's reduction ends with the cross-GPU exchange (one kernel per GPU)"
        elif self.partial:
            nccl = combine_step(cfg, self.bufs, world)
            self.step = lambda: (self.go(), nccl())
            self.combine = "the KernelOp's reduction, then an NCCL all-reduce of the per-GPU results"

    def close(self):
        if self.xchg is not None:
            import torch
            torch.cuda.synchronize(self.local)
            st = self.xchg.status()
            torch.distributed.barrier()       # no peer stores into this GPU's buffer any more
            self.xchg.close()
            if st:
                raise RuntimeError(f"{self.cfg}: cross-GPU exchange status 0x{st:x} (a peer did not arrive in time)")
        self.mod.close()


def _timed(job, steps: int, warmup: int, world: int, rank: int, clocks_active: bool):
    """Device time of ``steps`` steps after ``warmup``: max over ranks, plus the clock record."""
    import torch
    local = job.local

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(warmup):
        job.step()
    torch.cuda.synchronize(local)
    st = job.mod.status()
    if st:
        raise RuntimeError(f"{job.cfg}: kernel status 0x{st:x} during warm-up")
    clocks = ClockSampler(list(range(min(world, torch.cuda.device_count()))) if world > 1 else [local],
                          active=clocks_active and rank == 0)
    # inputs smaller than L2 would stay cached across steps: each step then runs
    # after a write of a buffer larger than L2 and is timed by its own events
    footprint = sum(t.numel() * t.element_size() for t in job.bufs.values())
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=job.device) if footprint < L2_BYTES else None
    barrier()
    torch.cuda.synchronize(local)
    clocks.start()
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            job.step()
        e1.record()
        torch.cuda.synchronize(local)
        timed_ms = e0.elapsed_time(e1)
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for a, b in ev:
            flush.fill_(1)
            a.record()
            job.step()
            b.record()
        torch.cuda.synchronize(local)
        timed_ms = sum(a.elapsed_time(b) for a, b in ev)
    clocks.stop()
    barrier()
    # a timed region of a few milliseconds gives the poller one or two samples: run the
    # same steps again for about 0.2 s, untimed, and sample the clocks over that pass too
    clock_pass = None
    ms_max = max_over_ranks(timed_ms, world, job.device)     # every rank: the same pass length below
    if ms_max < 100.0 and flush is None:
        reps = min(20000, max(steps, int(200.0 / max(ms_max / steps, 1e-3))))
        pass2 = ClockSampler(list(range(min(world, torch.cuda.device_count()))) if world > 1 else [local],
                             active=clocks_active and rank == 0)
        torch.cuda.synchronize(local)
        pass2.start()
        for _ in range(reps):
            job.step()
        torch.cuda.synchronize(local)
        pass2.stop()
        barrier()
        clock_pass = dict(pass2.summary(), steps=reps, note="the same steps again, untimed, right after the timed "
                                                           "region, so that the clock record has enough samples")
        pass2.close()
    clocks.close()
    st = job.mod.status()
    if st:
        raise RuntimeError(f"{job.cfg}: kernel status 0x{st:x} in the timed region")
    l2 = ("inputs larger than L2 (126 MB), no flush needed" if flush is None else
          f"working set {footprint} B < L2: a {L2_FLUSH_BYTES >> 20} MiB buffer is written before every "
          "timed step, and each step is timed by its own CUDA events")
    record = clocks.summary()
    if clock_pass is not None:
        record["second_pass"] = clock_pass
    return ms_max, record, l2


def _e2e(job, steps: int, world: int) -> dict:
    """The same metric through the C-ABI host-buffer call (emmy_run_host):
    pinned host inputs copied in and outputs copied out inside the timed
    region, every step."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    nbytes, roles, ptrs, host = [], [], [], {}
    for name in job.spec.arg_order:
        t = job.bufs[name]
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        out = job.spec.args[name].get("output")
        if not out:
            h.copy_(t)
        host[name] = h
        ptrs.append(h.data_ptr())
        nbytes.append(h.numel() * h.element_size())
        roles.append(runtime.EMMY_ROLE_OUT if out else runtime.EMMY_ROLE_IN)
    job.mod.run_host(ptrs, nbytes, roles, stream=job.stream)  # warm the module's device buffers
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(job.local)
    t0 = time.perf_counter()
    for _ in range(steps):
        job.mod.run_host(ptrs, nbytes, roles, stream=job.stream)
        if job.partial:
            # the per-GPU partials of the host call's output are combined on the host's behalf
            host_out = host[job.spec.outputs[0]]
            part = host_out.to(job.device)
            torch.distributed.all_reduce(part, op=torch.distributed.ReduceOp.SUM)
            host_out.copy_(part)
    el = max_over_ranks(time.perf_counter() - t0, world, job.device)
    h2d = sum(b for b, r in zip(nbytes, roles) if r == runtime.EMMY_ROLE_IN)
    d2h = sum(b for b, r in zip(nbytes, roles) if r == runtime.EMMY_ROLE_OUT)
    latency = job.unit == "us"
    units = job.units * (world if job.mode == "weak" else 1)
    value = el / steps * 1e6 if latency else units * steps / el / _units_scale(job.unit)
    return {"value": round(value, 3), "unit": job.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "path": "emmy_run_host (C ABI) on pinned host buffers"
            + (", per rank on its shard" if world > 1 else "")}


def _verify(job) -> dict:
    """The job checks its own result (multi-GPU runs): sharded outputs bit-equal
    to the whole-problem kernel on sampled rows (pointwise, GEMM: the same
    module's unit-range launch on those rows), row maxima exact and row sums
    within rtol 1e-5 of an f64 sum (row reductions), and the combined total
    of a full-array sum within rtol 1e-5 of an f64 checksum over all GPUs."""
    import torch
    from emmy_ptx_compiler_b200 import compiler, runtime
    cfg, sh = job.cfg, job.shard
    if sh is None:
        return {"checked": False}
    torch.cuda.synchronize(job.local)
    if cfg == "c4":
        part = job.bufs["x"].double().sum().reshape(1)
        torch.distributed.all_reduce(part, op=torch.distributed.ReduceOp.SUM)
        got, want = float(job.bufs["sum_1"].double().item()), float(part.item())
        ok = abs(got - want) <= 1e-5 * abs(want) + 0.05
        return {"checked": True, "ok": bool(ok), "what": "combined total vs f64 checksum of all shards, rtol 1e-5",
                "total": got, "f64": want}
    if cfg == "c3":
        x = job.bufs["x"]
        mx_ok = bool(torch.equal(job.bufs["max_1"], x.max(dim=1).values))
        ref = x.double().sum(dim=1)
        err = (job.bufs["sum_1"].double() - ref).abs()
        s_ok = bool((err <= 1e-5 * ref.abs() + 1e-3).all())
        return {"checked": True, "ok": mx_ok and s_ok, "what": "row maxima exact; row sums vs f64 within rtol 1e-5",
                "rows": int(x.shape[0])}
    # pointwise / GEMM: the whole-problem module over the first and the last aligned block of
    # this shard's units (unit-range launches), against the shard kernel's output there
    bundle = compiler.compile_bundle(job.spec.ir_path, want_cubin=True)
    full = runtime.Module(bundle["cubin"], job.spec.entry, job.local)
    total, align, per_unit = full.unit_range()
    upr = total // sh.extent                       # units per row of the sharded axis
    u0, u1 = sh.lo * upr, sh.hi * upr              # this shard's units
    blocks = []
    if u0 % align == 0 and u1 - u0 >= align:
        blocks = sorted({(u0, u0 + align), ((u1 // align - 1) * align, (u1 // align) * align)})
    ok, checked = True, []
    out = job.spec.outputs[0]
    for b, e in blocks:
        words, tmp = [], None
        for name, t, pb in zip(job.spec.arg_order, job.order, per_unit):
            if name in sh.buffers and pb:
                if name == out:
                    tmp = torch.empty(((e - b) * pb + t.element_size() - 1) // t.element_size(),
                                      dtype=t.dtype, device=t.device)
                    words.append(tmp.data_ptr() - b * pb)
                else:
                    words.append(t.data_ptr() - u0 * pb)
            else:
                words.append(t.data_ptr())
        full.launch_range(words, b, e, stream=job.stream)
        torch.cuda.synchronize(job.local)
        pb = per_unit[job.spec.arg_order.index(out)]
        mine = job.bufs[out].view(-1).view(torch.uint8)[(b - u0) * pb:(e - u0) * pb]
        same = bool(torch.equal(tmp.view(torch.uint8)[:(e - b) * pb], mine))
        ok = ok and same
        checked.append([b, e])
    full.close()
    return {"checked": bool(checked), "ok": ok, "unit_blocks": checked,
            "what": "shard output bit-equal to the whole-problem kernel (unit-range launches) on the first and "
                    "last aligned block of the shard's units"}


def measure(cfg: str, args, rank: int, world: int, local: int, mode: str, *, extras: bool = True,
            combine: str = "fused") -> dict:
    """One config: device-timed value, roofline, e2e, and (rank 0, N = 1) the
    reference-PTX and CPU baselines."""
    job = Job(cfg, rank, world, local, mode, combine)
    try:
        ms_max, clocks, l2 = _timed(job, args.steps, args.warmup, world, rank, clocks_active=True)
        check = _verify(job) if world > 1 and mode == "strong" else None
        latency = job.unit == "us"
        per_launch_ms = ms_max / args.steps
        scale = 1 if latency else _units_scale(job.unit)
        job_units = job.units * (world if mode == "weak" else 1)
        if latency:
            value = achieved = per_launch_ms * 1e3
        else:
            value = job_units * args.steps / (ms_max / 1e3) / scale
            # per GPU: the units one launch processes on the slowest rank
            achieved = job_units / world / (per_launch_ms / 1e3) / scale
        e2e_steps = max(1, args.steps if latency else min(args.steps, 5))
        e2e = _e2e(job, e2e_steps, world) if extras else None
        ref_ptx = cpu = None
        if rank == 0 and world == 1 and extras:
            if not args.no_ref_ptx:
                ref_ptx = time_reference_ptx(cfg, job, job.local, job.units, job.unit)
            if not args.no_cpu_baseline:
                cpu = cpu_baseline(cfg, seconds=args.cpu_seconds if cfg == args.config else args.cpu_seconds / 2)
        graph = latency_extras(job, args) if latency and extras else None
    finally:
        job.close()
    pk, pk_kind = peaks()
    bound = job.bound
    peak = pk["hbm_gbs"] if bound == "hbm" else pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    if bound == "fp32":
        peak, pk_kind = round(FP32_NOMINAL_TFLOPS, 1), "nominal"
    if bound == "tf32x3":
        peak, pk_kind = round(TF32_NOMINAL_TFLOPS / 3, 1), "nominal"
    peak_key = {"hbm": "hbm_gbs", "tensor": "bf16_tflops (burst: one kernel timed alone)",
                "fp32": "fp32 CUDA cores", "latency": "none",
                "tf32x3": "dense tf32 tensor peak / 3 (three MMAs per f32 product)"}[bound]
    traffic = DRAM_TRAFFIC.get(job.case_id) if world == 1 else None
    entry = {
        "value": round(value, 2), "unit": job.unit, "ms_per_step": round(per_launch_ms, 4),
        "workload": job.workload, "case": job.case_id, "launch": job.launch, "l2": l2,
        "roofline": ({"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": job.unit,
                      "frac": round(achieved / peak, 4), "traffic": traffic,
                      "peak_source": f"{pk_kind} ({peak_key})", "units_per_launch": job_units // world,
                      "per": "GPU (slowest rank)"} if not latency else
                     {"bound": "latency", "achieved": round(achieved, 3), "peak": None, "unit": "us", "frac": None,
                      "traffic": None, "units_per_launch": job.units,
                      "note": "768 bytes per launch: bounded by launch latency, not by HBM or tensor cores"}),
        "clocks": clocks,
        "gpu_launches": args.steps,
    }
    if bound == "tensor" and not latency:
        entry["roofline"]["frac_of_sustained"] = round(achieved / pk.get("bf16_tflops_sustained",
                                                                          FALLBACK_PEAKS["bf16_tflops_sustained"]), 4)
    if e2e is not None:
        entry["e2e"] = e2e
    if ref_ptx is not None:
        entry["reference_ptx_gpu"] = ref_ptx
    if cpu is not None:
        entry["cpu_baseline"] = cpu
    if graph is not None:
        entry["latency"] = graph
    if check is not None:
        entry["check"] = check
    if world > 1:
        sh = job.shard
        entry["parallelism"] = (
            f"strong scaling: the BASELINE problem split over {world} ranks, rows [lo, hi) of axis "
            f"'{sh.axis}' ({sh.extent // world} of {sh.extent}) per rank"
            + (f"; per-rank results combined inside every step: {job.combine}"
               if sh.mode == "partial" else "; no collective") if mode == "strong" else
            f"weak scaling: {world} ranks, each its own full-size copy of the problem; "
            + ("per-rank sums combined by an NCCL all-reduce in every step" if cfg == "c4" else "no collective"))
    return entry


def latency_extras(job, args) -> dict:
    """C1: back-to-back launch rate, and the same launches replayed as a CUDA graph."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    local = job.local
    torch.cuda.synchronize(local)
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    for _ in range(args.steps):
        job.go()
    b1.record()
    torch.cuda.synchronize(local)
    back_to_back_us = b0.elapsed_time(b1) * 1e3 / args.steps
    gs = torch.cuda.Stream(device=local)
    torch.cuda.synchronize(local)
    with runtime.Graph.record(local, gs.cuda_stream) as g:
        for _ in range(args.steps):
            job.mod.launch(job.order, stream=gs.cuda_stream)
    for _ in range(args.warmup):
        g.launch(gs.cuda_stream)
    torch.cuda.synchronize(local)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(gs)
    g.launch(gs.cuda_stream)
    g1.record(gs)
    torch.cuda.synchronize(local)
    out = {"graph_replay_us_per_launch": round(g0.elapsed_time(g1) * 1e3 / args.steps, 3),
           "launches_per_graph": args.steps, "graph_path": "emmy_graph_begin/end/launch (C ABI)",
           "back_to_back_us_per_launch": round(back_to_back_us, 3),
           "note": "value: one launch timed alone after an L2 flush; the back-to-back and graph "
                   "figures run with L2 warm"}
    g.close()
    return out


def run_ours(args, rank: int, world: int, local: int) -> dict | None:
    import torch
    torch.cuda.set_device(local)
    mode = "strong" if world > 1 else "single"
    main_cfg = args.config
    entry = measure(main_cfg, args, rank, world, local, mode)
    weak = None
    if world > 1 and not args.only:
        weak = measure(main_cfg, args, rank, world, local, "weak", extras=False)
    others = {}
    if main_cfg == "c2" and not args.only:
        for cfg in ("c3", "c4", "c5"):
            others[cfg] = measure(cfg, args, rank, world, local, mode)
            if world > 1 and cfg == "c4":
                # the same step with the combine as a separate NCCL all-reduce, and weak scaling
                others[cfg]["combine_nccl"] = {k: v for k, v in measure(cfg, args, rank, world, local, mode,
                                                                        extras=False, combine="nccl").items()
                                               if k in ("value", "unit", "ms_per_step", "parallelism")}
                others[cfg]["weak"] = {k: v for k, v in measure(cfg, args, rank, world, local, "weak",
                                                                 extras=False).items()
                                       if k in ("value", "unit", "ms_per_step", "parallelism")}
    if rank != 0:
        return None
    latency = entry["unit"] == "us"
    dtype = {"c5": "bf16"}.get(main_cfg, "f32")
    line = {
        "metric": METRIC, "value": entry["value"], "unit": entry["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": entry["ms_per_step"], "higher_is_better": not latency,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded on device, BASELINE distributions)",
        "config": {"workload": entry["workload"], "case": entry["case"],
                   "parallelism": entry.get("parallelism", "1 GPU"), "l2": entry["l2"], "launch": entry["launch"]},
        "roofline": entry["roofline"],
        "e2e": entry.get("e2e"),
        "gpu_launches": entry["gpu_launches"],
        "clocks": entry["clocks"],
    }
    for k in ("reference_ptx_gpu", "cpu_baseline", "latency", "check"):
        if k in entry:
            line[k] = entry[k]
    if weak is not None:
        line["weak"] = {k: weak[k] for k in ("value", "unit", "ms_per_step", "parallelism", "clocks")}
    if others:
        line["configs"] = others
        line["gpu_launches"] = args.steps * (1 + len(others))
        line["configs_note"] = ("C3-C5 of BASELINE, each timed like the headline line (same steps, warm-up and "
                                "timing rules) in the same process after it; gpu_launches counts every config's "
                                "timed launches")
    return line


def time_reference_ptx(cfg: str, job, local: int, units: int, unit: str) -> dict:
    """The reference compiler's own PTX for the same work on the same B200
    (JIT-loaded, meta.json launch), on the same device buffers.

    * c4: the reference indexes in s32 and cannot address 2^31 elements in
      one launch; its route is its 2^28-element IR launched 8 times over
      consecutive chunks (one step = the 8 launches);
    * c5: the reference cannot lower bf16 loads; its route is its f32 naive
      matmul IR on f32 copies of A and B, over the whole problem."""
    import torch
    from emmy_ptx_compiler_b200 import harness, runtime
    spec = job.spec
    stream = torch.cuda.current_stream(local).cuda_stream
    plan = []   # (module, args, grid, block, work units of this launch)
    mods = []
    if cfg == "c4":
        rdir = CASES / "c4_sum_chunk_2p28"
        rs = harness.load_case(rdir)
        m = runtime.Module((rdir / "ref.ptx").read_bytes(), rs.entry, local)
        mods.append(m)
        x, chunk = job.bufs["x"], rs.args["x"]["shape"][0]
        parts = torch.zeros(x.numel() // chunk, dtype=torch.float32, device=job.device)
        for c in range(x.numel() // chunk):
            plan.append((m, [x[c * chunk:(c + 1) * chunk], parts[c:c + 1]], rs.kernel["grid"], rs.kernel["block"]))
        route = f"{len(plan)} launches of the reference's {chunk}-element full-sum IR over consecutive chunks"
        work = units
    elif cfg == "c5":
        rdir = CASES / "c5_gemm_full" / "ref_f32"
        rs = harness.load_case(rdir)
        m = runtime.Module((rdir / "ref.ptx").read_bytes(), rs.entry, local)
        mods.append(m)
        A, B = job.bufs["A"].float(), job.bufs["B"].float()
        out = torch.zeros((A.shape[0], B.shape[1]), dtype=torch.float32, device=job.device)
        plan.append((m, [A, B, job.bufs["bias"], out], rs.kernel["grid"], rs.kernel["block"]))
        route = "the reference's f32 naive matmul IR on f32 copies of A and B (it cannot lower bf16 loads)"
        work = units
    else:
        ref = spec.root / "ref.ptx"
        if not ref.is_file():
            return {"unavailable": "no reference PTX for this IR"}
        m = runtime.Module(ref.read_bytes(), spec.entry, local)
        mods.append(m)
        plan.append((m, [job.bufs[n] for n in spec.arg_order], spec.kernel["grid"], spec.kernel["block"]))
        route = "the reference compiler's PTX for the same IR, meta.json launch"
        work = units

    def one():
        for m, a, g, b in plan:
            m.launch(a, stream=stream, grid=g, block=b)

    for _ in range(1 if cfg in ("c4", "c5") else 3):
        one()
    torch.cuda.synchronize(local)
    n = 50 if unit == "us" else (2 if cfg in ("c4", "c5") else 5)
    footprint = sum(t.numel() * t.element_size() for t in job.bufs.values())
    flush = (torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=job.device)
             if footprint < L2_BYTES else None)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for e0, e1 in ev:    # same rule as our arm: an L2 flush before each launch of a small working set
        if flush is not None:
            flush.fill_(1)
        e0.record()
        one()
        e1.record()
    torch.cuda.synchronize(local)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / n
    for m in mods:
        m.close()
    value = ms * 1e3 if unit == "us" else work / (ms / 1e3) / _units_scale(unit)
    return {"value": round(value, 3), "unit": unit, "ms_per_step": round(ms, 4), "route": route,
            "launch": {"grid": plan[0][2], "block": plan[0][3]}, "launches_per_step": len(plan)}


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
    ap.add_argument("--only", action="store_true",
                    help="time only --config (no C3-C5 block after C2, no weak-scaling pass at N > 1)")
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
