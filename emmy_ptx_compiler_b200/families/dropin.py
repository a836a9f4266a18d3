"""The drop-in entry: ``<KernelOp.name>`` with exactly the ``arg_order``
parameters, correct under the launch the reference's runner makes.

The reference's contract (compile.py:854-864, README.md:170-182) is one
``.visible .entry <KernelOp.name>`` whose parameters are the ``arg_order``
buffers, launched with meta.json's grid, block and ``smem_bytes``.  Some of
this backend's fast kernels take more than that: a unit range (two u64
words after the buffers) so that the C ABI can pipeline host copies and shard
launches, and, for the tcgen05 GEMM, two TMA tensor maps encoded on the host.
Such a module carries two entries:

* ``<name>__emmy`` - the fast kernel with its extra parameters, launched by
  libemmy_b200 with the geometry in the module's launch record;
* ``<name>`` - the drop-in, ``arg_order`` parameters only.  It runs the same
  fast code over the whole problem when launched with the launch record's
  block shape (and dynamic shared memory), and otherwise a path that is
  correct under any launch of the reference's contract:

  - pointwise kernels are correct under every launch (vector tiles under the
    record's 256-thread blocks, a scalar grid-stride loop under any other), so
    the drop-in always runs the module's body;
  - row-fused and attention kernels fall back to the IR's own schedule
    (the schedule family: the reference's thread model, compiled for
    sm_100a), which is what meta.json's geometry was written for; a fast
    kernel that needs a cooperative launch (CTAs that wait on one another)
    is never run from the drop-in;
  - the GEMM's drop-in is a separate kernel (families/gemm.py).

The PTX parameter names are nvcc's (``<entry>_param_<i>``), not the
reference's ``param_<name>``: a launch binds parameters by position, and
renaming them would mean editing compiler-written PTX.
"""

from __future__ import annotations

import re

from .. import ir
from ..errors import UnsupportedIR
from . import schedule
from .common import KernelSource, c_ident

NATIVE_SUFFIX = "__emmy"


def native_entry(name: str) -> str:
    return name + NATIVE_SUFFIX


def _header(source: str, name: str) -> re.Match:
    pat = re.compile(r'^extern "C" __global__ void (__launch_bounds__\([^)]*\) )?' + re.escape(name)
                     + r"\((?P<sig>.*)\) \{$", re.M)
    found = list(pat.finditer(source))
    if len(found) != 1:
        raise ValueError(f"expected one kernel header for {name}, found {len(found)}")
    return found[0]


def _param_name(decl: str) -> str:
    return decl.split()[-1].lstrip("*&")


def _threads(block) -> int:
    out = 1
    for x in tuple(block or ()) or (1,):
        out *= int(x)
    return out


def attach(ks: KernelSource, kop: ir.KernelOp, shapes: dict, dtypes: dict, args: list[str],
           scalars: dict, written: set, meta: dict | None) -> KernelSource:
    """Give a module whose fast kernel takes a unit range the drop-in entry
    (see the module docstring).  Modules whose kernel already takes exactly
    the ``arg_order`` parameters are returned unchanged."""
    if not ks.launch.range_total or ks.tmaps or "entries" in ks.notes:
        return ks
    name = ks.entry
    m = _header(ks.source, name)
    sig = [s.strip() for s in m.group("sig").split(",")]
    n = len(args)
    if len(sig) != n + 2:
        raise ValueError(f"{name}: {len(sig)} kernel parameters for {n} arg_order names + a unit range")
    body_fn = f"emmy_body_{c_ident(name)}"
    src = (ks.source[:m.start()] + f"static __device__ __forceinline__ void {body_fn}({m.group('sig')}) {{"
           + ks.source[m.end():])
    lb = m.group(1) or ""
    names = [_param_name(s) for s in sig]
    native = (f'extern "C" __global__ void {lb}{native_entry(name)}({", ".join(sig)}) {{\n'
              f"    {body_fn}({', '.join(names)});\n}}\n")
    whole = f"{body_fn}({', '.join(names[:n])}, 0ull, ~0ull);"
    meta = meta or {}
    meta_threads = _threads(meta.get("block")) if meta.get("block") else 0
    own = ks.launch.block
    threads = max(_threads(own), meta_threads)
    fallback = None
    if ks.family in ("rownorm", "attention"):
        try:
            plan = schedule.match(kop, shapes, dtypes)
            if plan is not None:
                fallback = schedule.generate(kop, plan, shapes, dtypes, args, scalars, written, meta,
                                             device_fn=f"emmy_sched_{c_ident(name)}")
        except UnsupportedIR:
            fallback = None
    lines = [src, native]
    cooperative = ks.launch.cooperative
    if cooperative and fallback is None:
        # no schedule to fall back on, and the fast body needs a cooperative launch: the
        # drop-in only reports that it cannot run (the C ABI launches the fast entry)
        lines.append(
            f'extern "C" __global__ void {name}({", ".join(sig[:n])}) {{\n'
            "    if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0 && blockIdx.x == 0 &&\n"
            "        blockIdx.y == 0 && blockIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);\n}\n")
        mode = "reports EMMY_STATUS_BAD_LAUNCH (the fast kernel needs a cooperative launch; no schedule to run)"
    elif fallback is None:
        lines.append(f'extern "C" __global__ void __launch_bounds__({threads}) {name}({", ".join(sig[:n])}) {{\n'
                     f"    {whole}\n}}\n")
        mode = "fast body under every launch" if ks.family == "pointwise" else \
            "fast body; other launches raise EMMY_STATUS_BAD_LAUNCH"
    elif cooperative:
        # the fast kernel's CTAs wait on one another, which only a cooperative launch makes safe,
        # and a kernel cannot tell how it was launched: the drop-in always runs the IR's schedule
        lines.append(fallback.source)
        threads = max(threads, 1024 if not meta_threads else meta_threads)
        lines.append(
            f'extern "C" __global__ void __launch_bounds__({threads}) {name}({", ".join(sig[:n])}) {{\n'
            f"    emmy_sched_{c_ident(name)}({', '.join(names[:n])});\n}}\n")
        mode = "the IR's own schedule under every launch (the fast kernel needs a cooperative launch)"
    else:
        lines.append(fallback.source)
        threads = max(threads, 1024 if not meta_threads else meta_threads)
        lines.append(
            f'extern "C" __global__ void __launch_bounds__({threads}) {name}({", ".join(sig[:n])}) {{\n'
            "    uint32_t emmy_dyn;\n"
            '    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(emmy_dyn));\n'
            + (f"    uint32_t emmy_ncl;\n"
               '    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(emmy_ncl));\n'
               if ks.launch.cluster[0] > 1 else "") +
            f"    if (blockDim.x == {own[0]} && blockDim.y == {own[1]} && blockDim.z == {own[2]}"
            f" && emmy_dyn >= {ks.launch.smem}u"
            + (f" && emmy_ncl == {ks.launch.cluster[0]}u" if ks.launch.cluster[0] > 1 else "") + ") {\n"
            f"        {whole}\n"
            "    } else {\n"
            f"        emmy_sched_{c_ident(name)}({', '.join(names[:n])});\n"
            "    }\n}\n")
        mode = "fast body under the launch record's block shape, else the IR's own schedule"
    notes = dict(ks.notes)
    notes["entries"] = {"drop_in": name, "native": native_entry(name), "drop_in_path": mode}
    return KernelSource(entry=name, source="\n".join(lines), launch=ks.launch, params=ks.params,
                        family=ks.family, notes=notes, tmaps=ks.tmaps)
