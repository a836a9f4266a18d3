"""Drop-in compiler surface: ``compile_ir``, ``compile_bundle``, ``Compiler``, ``main``.

Mirrors the reference's L1 entry points (compile.py:3164-3227):

* ``python compile.py kernel.ir.json > out.ptx`` prints one PTX module,
  ASCII only, with one ``.visible .entry <KernelOp.name>`` whose parameters
  are the ``meta.json`` ``arg_order`` buffers (``.u64`` pointers, or typed
  scalars for ``args[i].scalar``), now ``.target sm_100a``;
* wrong usage prints the usage line and exits 2; an IR this backend cannot
  lower prints ``unsupported ...`` on stderr and exits 2 (compile.py:1516-1518);
* ``compile_bundle`` returns the reference's keys (``ptx, entry, args, shapes,
  dtypes, smem_bytes, dynamic_smem, block, virt_regs, stats, ops, ir_txt,
  meta, bytes``) plus ``family``, ``launch`` (the geometry the module is
  tuned for), ``source`` (generated CUDA) and ``notes``.

Lowering replaces the reference's PTX printer (compile.py:342-3161): the
KernelOp is classified into one of three hand-written sm_100a families,
which emit specialised CUDA C++ that nvcc compiles.
"""

from __future__ import annotations

import json
import sys
from dataclasses import dataclass
from pathlib import Path

from . import frontend, ir, toolchain
from .errors import ToolchainError, UnsupportedIR
from .families import attention, canon, dropin, gemm, pointwise, reduction, rownorm, schedule
from .families.common import KernelSource


@dataclass
class Lowered:
    kernel: KernelSource
    args: list[str]
    shapes: dict
    dtypes: dict
    meta: dict


def _scalars(meta: dict | None, dtypes: dict) -> dict[str, str]:
    out: dict[str, str] = {}
    for arg in (meta or {}).get("args") or []:
        if arg.get("scalar"):
            dt = ir.canon_dtype(arg.get("dtype") or dtypes.get(arg.get("name")))
            out[arg["name"]] = "f32" if dt == "f32" else "i32"
    return out


def _pointwise_tune(tune: dict | None) -> dict:
    """The pointwise generator's schedule knobs a caller may set (every value
    gives the same results)."""
    tune = dict(tune or {})
    bad = set(tune) - {"unroll", "pipeline", "min_blocks", "order", "tile_u"}
    if bad:
        raise ValueError(f"unknown pointwise_tune keys: {sorted(bad)}")
    return tune


def lower(kop: ir.KernelOp, shapes: dict, dtypes: dict, args: list[str], meta: dict | None,
          options: dict | None = None) -> Lowered:
    """Classify ``kop`` into a family and generate its specialised source.

    ``options`` selects among equivalent schedules (results do not depend on
    it): ``{"gemm_variant": "auto" | "pair" | "single", "gemm_tune": {...}
    (families/gemm.py PAIR_TUNE),
    "pointwise_pair": "auto" | True | False, "pointwise_tune": {"unroll", "pipeline",
    "min_blocks", "order", "tile_u"}, "attention_first_pass": "auto" | "tiled",
    "attention_kernel": "auto" | "tc" | "exact", "attention_exchange": "auto" | "cluster" | "grid",
    "attention_tune": {...} (families/attention_tc.py TC_TUNE),
    "family": "schedule"}``; the
    last skips the fast families.  A KernelOp no fast family takes (or one a
    family recognises but cannot specialise) keeps its own schedule."""
    meta = meta or {}
    options = options or {}
    written = {s.output for s in ir.walk(kop.body) if isinstance(s, ir.Write)}
    scalars = _scalars(meta, dtypes)
    for name in args:
        if name not in scalars and name not in shapes and name not in dtypes:
            raise UnsupportedIR(f"parameter {name!r} has no shape or dtype")
    if options.get("family") == "schedule":
        plan = schedule.match(kop, shapes, dtypes)
        if plan is None:
            raise UnsupportedIR(f"KernelOp {kop.name!r} cannot be lowered as its own schedule "
                                f"(unsupported nodes: {', '.join(schedule.unsupported_nodes(kop)) or 'layout'})")
        ks = schedule.generate(kop, plan, shapes, dtypes, args, scalars, written, meta)
        return Lowered(ks, args, shapes, dtypes, meta)
    meta_threads = dropin._threads(meta.get("block")) if meta.get("block") else 0
    # a matmul staged through shared memory is still a matmul: prove it and lower the naive form
    staged = canon.staged_matmul(kop, shapes, dtypes, meta)
    if staged is not None:
        try:
            plan = gemm.match(staged, shapes, dtypes)
            if plan is not None:
                ks = gemm.generate(staged, plan, shapes, dtypes, args, scalars, written,
                                   variant=options.get("gemm_variant", "auto"), meta_threads=meta_threads,
                                   tune=options.get("gemm_tune"))
                ks.notes["canonical_form"] = "staged matmul -> naive matmul"
                return Lowered(ks, args, shapes, dtypes, meta)
        except UnsupportedIR:
            pass
    fast = (
        ("attention", lambda: attention.match(kop, shapes, dtypes),
         lambda pl: attention.generate(kop, pl, shapes, dtypes, args, scalars, written,
                                       first_pass=options.get("attention_first_pass", "auto"),
                                       kernel=options.get("attention_kernel", "auto"),
                                       exchange=options.get("attention_exchange", "auto"),
                                       tune=options.get("attention_tune"))),
        ("gemm", lambda: gemm.match(kop, shapes, dtypes),
         lambda pl: gemm.generate(kop, pl, shapes, dtypes, args, scalars, written,
                                  variant=options.get("gemm_variant", "auto"), meta_threads=meta_threads,
                                  tune=options.get("gemm_tune"))),
        ("reduction", lambda: reduction.match(kop, shapes, dtypes),
         lambda pl: reduction.generate(kop, pl, shapes, dtypes, args, scalars, written)),
        ("rownorm", lambda: rownorm.match(kop, shapes, dtypes),
         lambda pl: rownorm.generate(kop, pl, shapes, dtypes, args, scalars, written)),
        ("pointwise", lambda: pointwise.match(kop),
         lambda pl: pointwise.generate(kop, pl, shapes, dtypes, args, scalars, written,
                                       pair=options.get("pointwise_pair", "auto"),
                                       **_pointwise_tune(options.get("pointwise_tune")))),
    )
    rejected: list[str] = []
    for fam, match, generate in fast:
        try:
            plan = match()
            if plan is None:
                continue
            ks = dropin.attach(generate(plan), kop, shapes, dtypes, args, scalars, written, meta)
            return Lowered(ks, args, shapes, dtypes, meta)
        except UnsupportedIR as exc:
            # a family that recognised the shape but cannot specialise it (dtype,
            # head size, memory access pattern ...): the schedule family takes it
            rejected.append(f"{fam}: {exc}")
    # no recognised computation: keep the schedule the IR spells out
    plan = schedule.match(kop, shapes, dtypes)
    if plan is not None:
        ks = schedule.generate(kop, plan, shapes, dtypes, args, scalars, written, meta)
        return Lowered(ks, args, shapes, dtypes, meta)
    bad = schedule.unsupported_nodes(kop)
    kinds = sorted({type(s).__name__ for s in ir.walk(kop.body)})
    raise UnsupportedIR(f"KernelOp {kop.name!r} has nodes no sm_100a lowering supports "
                        f"({', '.join(bad) or 'layout'}; nodes: {', '.join(kinds)})"
                        + (f"; {'; '.join(rejected)}" if rejected else ""))


class Compiler:
    """``Compiler(kop, shapes, dtypes, args, meta).run() -> ptx``, the
    constructor the reference's tests use (compile.py:410-411, 823)."""

    def __init__(self, kop: ir.KernelOp, shapes: dict, dtypes: dict, args: list[str],
                 meta: dict | None = None, options: dict | None = None):
        self.kop = kop
        self.shapes = {k: tuple(int(x) for x in v) for k, v in shapes.items()}
        self.dtypes = dict(dtypes)
        self.args = list(args)
        self.meta = meta or {}
        self.options = dict(options or {})
        self.lowered: Lowered | None = None

    def lower(self) -> Lowered:
        if self.lowered is None:
            self.lowered = lower(self.kop, self.shapes, self.dtypes, self.args, self.meta, self.options)
        return self.lowered

    def run(self) -> str:
        ks = self.lower().kernel
        return toolchain.build(ks.source, "ptx", name=ks.entry).decode("ascii")

    def cubin(self) -> bytes:
        ks = self.lower().kernel
        return toolchain.build(ks.source, "cubin", name=ks.entry)


def _bundle_from(kop: ir.KernelOp, raw: dict | None, meta_k: dict | None, path: Path | None,
                 want_cubin: bool = False, options: dict | None = None) -> dict:
    args = frontend.arg_order_for(kop, meta_k)
    shapes, dtypes = frontend.load_shapes(raw, kop, meta_k)
    comp = Compiler(kop, shapes, dtypes, args, meta_k, options)
    low = comp.lower()
    ks = low.kernel
    ptx = comp.run()
    ir_txt = ""
    if path is not None:
        for cand in (path.with_suffix(".txt"), path.parent / (path.stem + ".ir.txt")):
            if cand.is_file():
                ir_txt = cand.read_text(encoding="utf-8")
                break
    mix: dict[str, int] = {}
    out = {
        "ptx": ptx,
        "entry": kop.name,
        "args": args,
        "shapes": {k: list(v) for k, v in shapes.items()},
        "dtypes": dtypes,
        "smem_bytes": ks.launch.smem,
        "dynamic_smem": ks.launch.smem > 48 * 1024,
        "block": ks.launch.block[0] * ks.launch.block[1] * ks.launch.block[2],
        # physical registers per entry from ptxas (the reference counted its virtual
        # registers by type; nvcc's PTX is not read here, so ptxas -v gives the counts)
        "virt_regs": _register_counts(ks),
        "stats": {"family": ks.family, **{k: v for k, v in ks.notes.items() if isinstance(v, (int, bool))}},
        "ops": mix,
        "ir_txt": ir_txt,
        "meta": meta_k or {},
        "bytes": len(ptx.encode("ascii", "replace")),
        "family": ks.family,
        "launch": {"grid": list(ks.launch.grid), "block": list(ks.launch.block), "smem": ks.launch.smem},
        "params": [{"name": p.name, "kind": p.kind, "dtype": p.dtype} for p in ks.params],
        "source": ks.source,
        "notes": ks.notes,
    }
    if want_cubin:
        out["cubin"] = comp.cubin()
    return out


def _register_counts(ks: KernelSource) -> dict:
    try:
        per = toolchain.register_usage(ks.source, ks.entry)
    except ToolchainError as exc:
        return {"unavailable": str(exc)[:200]}
    entry = per.get(ks.entry, {})
    return {"registers": entry.get("registers"), "spill_stores": entry.get("spill_stores", 0),
            "spill_loads": entry.get("spill_loads", 0), "entries": per, "source": "ptxas -v, sm_100a"}


def compile_bundle(path, want_cubin: bool = False, options: dict | None = None) -> dict:
    path = Path(path)
    raw = json.loads(path.read_text(encoding="utf-8"))
    info = frontend.load_graph(raw)
    meta_k = frontend.load_meta_kernel(path, info.kop.name)
    return _bundle_from(info.kop, raw, meta_k, path, want_cubin, options)


def compile_ir(path) -> str:
    return compile_bundle(path)["ptx"]


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv if argv is None else argv)
    if len(argv) != 2:
        print("usage: python compile.py path/to/kernel.ir.json", file=sys.stderr)
        return 2
    try:
        ptx = compile_ir(Path(argv[1]))
    except UnsupportedIR as exc:
        print(f"unsupported: {exc}", file=sys.stderr)
        return 2
    except ToolchainError as exc:
        print(f"toolchain error: {exc}", file=sys.stderr)
        return 3
    sys.stdout.write(ptx)
    return 0
