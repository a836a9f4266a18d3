"""Run a KernelOp fixture directory (IR JSON + meta.json) on a B200.

The reference's runner contract (README.md:170-182, meta written at
tools/make_proxy_set.py:75-86): inputs per ``args[]``, outputs listed in
``zero_outputs`` zero-filled before the launch, the entry launched with its
parameters in ``arg_order``.  Device buffers are torch tensors (PyTorch is
the allocator here); launches go through ``libemmy_b200`` on torch's
current stream, so torch CUDA events time them.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import compiler, runtime

TORCH_DTYPES = {"f32": "float32", "bf16": "bfloat16", "f16": "float16", "i32": "int32"}


def _torch():
    import torch
    return torch


@dataclass
class CaseSpec:
    root: Path
    ir_path: Path
    meta: dict
    kernel: dict

    @property
    def entry(self) -> str:
        return self.kernel["entry"]

    @property
    def arg_order(self) -> list[str]:
        return list(self.kernel["arg_order"])

    @property
    def args(self) -> dict[str, dict]:
        return {a["name"]: a for a in self.kernel.get("args") or []}

    @property
    def outputs(self) -> list[str]:
        return [a["name"] for a in self.kernel.get("args") or [] if a.get("output")]


def load_case(case_dir) -> CaseSpec:
    root = Path(case_dir)
    ir_path = next(root.glob("*.ir.json"))
    meta = json.loads((root / "meta.json").read_text())
    return CaseSpec(root, ir_path, meta, meta["kernels"][0])


def to_device(arr: np.ndarray, dtype: str, device: int = 0):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(arr, np.float32))
    tdt = getattr(torch, TORCH_DTYPES.get(dtype, "float32"))
    return t.to(device=f"cuda:{device}").to(tdt).contiguous()


def from_device(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()


class DeviceCase:
    """A fixture compiled by our backend and loaded on ``device``."""

    def __init__(self, case_dir, device: int = 0, options: dict | None = None):
        self.spec = load_case(case_dir)
        self.device = device
        self.bundle = compiler.compile_bundle(self.spec.ir_path, want_cubin=True, options=options)
        self.module = runtime.Module(self.bundle["cubin"], self.spec.entry, device)

    def buffers(self, inputs: dict[str, np.ndarray]) -> dict:
        """Device tensors for every parameter (outputs zero-filled)."""
        torch = _torch()
        out = {}
        for name in self.spec.arg_order:
            a = self.spec.args.get(name, {})
            dt = a.get("dtype") or self.bundle["dtypes"].get(name, "f32")
            if a.get("output"):
                shape = tuple(a.get("shape") or ()) or (1,)
                tdt = getattr(torch, TORCH_DTYPES.get(dt, "float32"))
                out[name] = torch.zeros(shape, dtype=tdt, device=f"cuda:{self.device}")
            else:
                out[name] = to_device(inputs[name], dt, self.device)
        return out

    def launch(self, bufs: dict, grid=None, block=None, stream: int | None = None) -> None:
        torch = _torch()
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        self.module.launch([bufs[n] for n in self.spec.arg_order], stream=stream, grid=grid, block=block)

    def run(self, inputs: dict[str, np.ndarray], grid=None, block=None) -> dict[str, np.ndarray]:
        torch = _torch()
        bufs = self.buffers(inputs)
        self.launch(bufs, grid, block)
        torch.cuda.synchronize(self.device)
        st = self.module.status()
        if st:
            raise runtime.EmmyError(-5, f"kernel status 0x{st:x}")
        return {n: from_device(bufs[n]) for n in self.spec.outputs}


class ForeignModule:
    """A PTX module not produced by this backend (e.g. the reference compiler's
    output), launched under the meta.json geometry as the reference runner did."""

    def __init__(self, ptx: bytes, spec: CaseSpec, device: int = 0):
        self.spec = spec
        self.device = device
        self.module = runtime.Module(ptx, spec.entry, device)

    def run(self, bufs: dict, chunks: list[tuple[int, int]] | None = None) -> None:
        """Launch once per (element offset, count) chunk of the first input
        (the s32-indexed reference cannot address 2^31 elements in one launch)."""
        torch = _torch()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        g, b = self.spec.kernel["grid"], self.spec.kernel["block"]
        smem = int(self.spec.kernel.get("smem_bytes") or 0)
        self.module.launch([bufs[n] for n in self.spec.arg_order], stream=stream, grid=g, block=b,
                           smem=smem if smem else None)


def _seeded_device_inputs(spec: CaseSpec, device: int, seed: int = 0) -> dict:
    """Device tensors with the fixture's shapes and input distributions."""
    torch = _torch()
    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(seed)
    bufs = {}
    for name in spec.arg_order:
        a = spec.args[name]
        shape = tuple(a.get("shape") or ()) or (1,)
        tdt = getattr(torch, TORCH_DTYPES.get(a.get("dtype", "f32"), "float32"))
        if a.get("output"):
            bufs[name] = torch.zeros(shape, dtype=tdt, device=f"cuda:{device}")
            continue
        init = a.get("init") or {"kind": "normal", "mean": 0.0, "std": 1.0}
        t = torch.empty(shape, dtype=torch.float32, device=f"cuda:{device}")
        if "data" in a:
            t.copy_(torch.tensor(a["data"], dtype=torch.float32).reshape(shape))
        elif init["kind"] == "uniform":
            t.uniform_(init["low"], init["high"], generator=g)
        else:
            t.normal_(init.get("mean", 0.0), init.get("std", 1.0), generator=g)
        bufs[name] = t.to(tdt)
    return bufs


def main(argv=None) -> int:
    """``python -m emmy_ptx_compiler_b200.harness CASE_DIR [--iters N] [--options JSON]``:
    compile a fixture (with lowering options, e.g. a GEMM tuning), launch it once
    and then N times on seeded device inputs, print the mean device time per
    launch (used for profiler captures of one kernel)."""
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("case_dir")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--options", default="{}", help="lowering options as JSON (compiler.lower)")
    ns = ap.parse_args(argv)
    torch = _torch()
    case = DeviceCase(ns.case_dir, ns.device, options=json.loads(ns.options))
    bufs = _seeded_device_inputs(case.spec, ns.device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    case.launch(bufs)
    torch.cuda.synchronize(ns.device)
    e0.record()
    for _ in range(ns.iters):
        case.launch(bufs)
    e1.record()
    torch.cuda.synchronize(ns.device)
    st = case.module.status()
    print(json.dumps({"case": case.spec.meta.get("id"), "family": case.module.family,
                      "ms_per_launch": e0.elapsed_time(e1) / ns.iters, "status": st,
                      "launch": {"grid": list(case.module.grid), "block": list(case.module.block),
                                 "smem": case.module.smem}}))
    case.module.close()
    return 1 if st else 0


if __name__ == "__main__":
    raise SystemExit(main())
