"""Pointwise family: one Tile cell = one independent element computation.

Replaces the reference's Tile lowering (compile.py:1520-1629), which runs one
cell per thread, guards leftover threads with ``bra SKIP`` and issues scalar
4-byte loads/stores unless the IR itself groups elements.  Here:

* cells are walked by a grid-stride loop sized to the machine (148 SMs), so
  any launch geometry computes the same result and no thread idles;
* when every Load/Write addresses the Tile axes directly (``x[a0, a1]``,
  broadcast forms like ``s[a1]`` or ``bias[a0]``, or a constant index) and
  the innermost extent is a multiple of 4, each thread moves 2 x 4
  consecutive cells per trip with 128-bit (f32) vector loads/stores, loads
  streamed with ``ld.global.cs``/``st.global.cs``;
* the fused op chain runs in registers through :mod:`..cgen`, with the
  reference's exact op semantics and FMA contraction sites;
* indices are 64-bit, so a Tile of 2^31 cells or more is one launch.

Anything else in the cell body (Conds with memory ops, multi-element Loads,
non-axis indices) takes the scalar grid-stride path with the same cell code.
"""

from __future__ import annotations

import functools
import math

from dataclasses import dataclass, field

from .. import ir
from ..ir import ELEM_BYTES
from ..cgen import DEVICE_PRELUDE, Emitter, ctype, load_to_kind, store_from
from .common import KernelSource, LaunchPlan, ParamSpec, SM_COUNT, launch_record_source
from .common import c_ident as _c

BLOCK = 256
UNROLL = 2
VEC = 4
PREFETCH = 0      # trips ahead to prefetch full-tile inputs into L2 (0 = off)
MIN_BLOCKS = 4    # __launch_bounds__ minimum blocks per SM (0 = compiler's choice)
# "tile" (default): each CTA takes TILE_U x BLOCK consecutive vectors, all loaded before any compute,
# and the grid follows the launch's range (C2, 2^28 cells: 6630 against 6303 GB/s for the
# persistent "grid" loop on the same GPU); "grid": persistent grid-stride vectors with a register
# double buffer; "blocked": each persistent CTA streams one contiguous chunk
ORDER = "tile"
TILE_U = 4        # 16 KiB of each streamed f32 input per CTA, 64 registers: 4 CTAs per SM
PIPELINE = True   # load the next trip's streamed vectors before computing the current trip
# bulk-copy pipeline: 8 consumer warps + 1 producer warp, 4096-cell tiles, up to 4 stages
BULK_MIN_CELLS = 1 << 20
BULK_CONSUMERS = 256
BULK_TILE = BULK_CONSUMERS * VEC * 4
BULK_SMEM_TARGET = 96 * 1024
BULK_CTAS_PER_SM = 2
_CELL_STMTS = (ir.Load, ir.Write, ir.Let, ir.Init, ir.Assign, ir.Accum, ir.Cond, ir.Select)


@dataclass
class PointwisePlan:
    tile: ir.Tile
    prelude: tuple  # statements before the Tile (none allowed today)
    axes: list[tuple[str, int]]
    ncells: int
    vector: bool
    reasons: list[str] = field(default_factory=list)
    pair: bool = False  # f32x2 lane pairs in the register-vector path


def _is_cell_body(body) -> bool:
    for s in ir.walk(body):
        if not isinstance(s, _CELL_STMTS):
            return False
        if isinstance(s, ir.Write) and s.atomic:
            return False
    return True


def match(kop: ir.KernelOp) -> PointwisePlan | None:
    body = ir.body_stmts(kop.body)
    tiles = [s for s in body if isinstance(s, ir.Tile)]
    if len(tiles) != 1 or len(body) != 1:
        return None
    tile = tiles[0]
    if not _is_cell_body(tile.body):
        return None
    if int(tile.aux_threads or 0):
        return None
    axes = [(a.name, a.size) for a in tile.axes]
    n = 1
    for _, e in axes:
        n *= e
    return PointwisePlan(tile=tile, prelude=(), axes=axes, ncells=n, vector=False)


def _axis_aligned(index, axes: list[tuple[str, int]]) -> list[int] | None:
    """Positions of the tile axes an index names, if it is exactly a tuple of
    axis variables in increasing axis order; None otherwise."""
    pos = {name: i for i, (name, _) in enumerate(axes)}
    out: list[int] = []
    for ix in index:
        if not isinstance(ix, ir.Var) or ix.name not in pos:
            return None
        p = pos[ix.name]
        if out and p <= out[-1]:
            return None
        out.append(p)
    return out


def _const_index(index) -> bool:
    return len(index) > 0 and all(isinstance(ix, ir.Literal) and not isinstance(ix.value, float)
                                  for ix in index)


def vector_eligible(plan: PointwisePlan, shapes: dict, dtypes: dict) -> tuple[bool, list[str]]:
    why: list[str] = []
    axes = plan.axes
    inner = axes[-1][1] if axes else 1
    if not axes or inner % VEC != 0:
        why.append(f"innermost extent {inner} is not a multiple of {VEC}")
    top = list(ir.body_stmts(plan.tile.body))
    for s in ir.walk(plan.tile.body):
        if isinstance(s, ir.Cond):
            for t in list(ir.walk(s.body)) + list(ir.walk(s.else_body)):
                if isinstance(t, (ir.Load, ir.Write)):
                    why.append("memory access under a Cond")
        if isinstance(s, ir.Load):
            if len(s.names) != 1:
                why.append(f"multi-element Load of {s.input}")
            elif not _const_index(s.index):
                pos = _axis_aligned(s.index, axes)
                shp = shapes.get(s.input)
                if pos is None:
                    why.append(f"Load {s.input} index is not a tile-axis tuple")
                elif shp is not None and tuple(shp) != tuple(axes[p][1] for p in pos):
                    why.append(f"Load {s.input} shape {shp} does not match its axes")
        if isinstance(s, ir.Write):
            pos = _axis_aligned(s.index, axes)
            shp = shapes.get(s.output)
            if len(s.values) != 1:
                why.append(f"multi-element Write of {s.output}")
            elif pos != list(range(len(axes))):
                why.append(f"Write {s.output} does not index every tile axis in order")
            elif shp is not None and tuple(shp) != tuple(e for _, e in axes):
                why.append(f"Write {s.output} shape {shp} does not match the tile")
    for s in top:
        if isinstance(s, (ir.Load, ir.Write)):
            dt = ir.canon_dtype((s.dtype if isinstance(s, ir.Load) else s.value_dtype)
                                or dtypes.get(s.input if isinstance(s, ir.Load) else s.output))
            if dt not in ("f32", "bf16", "f16"):
                why.append(f"element type {dt} has no vector form")
    return (not why), why


def _axis_strides(axes) -> list[int]:
    strides = [1] * len(axes)
    acc = 1
    for i in range(len(axes) - 1, -1, -1):
        strides[i] = acc
        acc *= axes[i][1]
    return strides


def _decode_axes(em: Emitter, axes, cell: str, prefix: str) -> None:
    strides = _axis_strides(axes)
    for i, ((name, ext), st) in enumerate(zip(axes, strides)):
        var = f"{prefix}{i}"
        q = cell if st == 1 else f"({cell} / {st}LL)"
        expr = q if i == 0 else f"({q} % {ext}LL)"
        if ext == 1:
            expr = "0LL"
        em.emit(f"const long long {var} = {expr};")
        em.bind_const(name, "int", var)


def _streamed_loads(plan: PointwisePlan) -> list[ir.Load]:
    """Loads that read every tile cell once (index = all tile axes in order)."""
    return [s for s in ir.walk(plan.tile.body)
            if isinstance(s, ir.Load) and not _const_index(s.index) and _streamed(s, plan)]


def generate(kop: ir.KernelOp, plan: PointwisePlan, shapes: dict, dtypes: dict, args: list[str],
             scalars: dict[str, str], written: set[str], *, variant: str = "auto",
             unroll: int = UNROLL, prefetch: int = PREFETCH, min_blocks: int = MIN_BLOCKS,
             order: str = ORDER, hoist_broadcast: bool = True, pair="auto",
             pipeline: bool = PIPELINE, tile_u: int = TILE_U) -> KernelSource:
    """``variant``: "auto"/"vector" (register vectors), or "bulk" (shared-memory
    ring fed by bulk async copies).  ``pair``: compute the cell body on two
    adjacent cells at once with packed f32x2 add/mul/fma ("auto": whenever the
    body is pure f32 arithmetic, see ``pairable``)."""
    vec_ok, why = vector_eligible(plan, shapes, dtypes)
    plan.vector = vec_ok
    plan.reasons = why
    streamed = _streamed_loads(plan) if vec_ok else []
    # measured on B200 (C2, 2^28 cells): register vectors 5.60 TB/s vs bulk pipeline 4.71 TB/s,
    # so "auto" keeps register vectors; the bulk pipeline stays selectable
    if streamed and variant == "bulk":
        return _generate_bulk(kop, plan, shapes, dtypes, args, scalars, written, streamed)
    params: list[ParamSpec] = []
    ptrs: dict[str, str] = {}
    sig: list[str] = []
    for name in args:
        if name in scalars:
            dt = scalars[name]
            sig.append(f"{ctype(dt)} p_{_c(name)}")
            params.append(ParamSpec(name, "scalar", dt))
            continue
        dt = ir.canon_dtype(dtypes.get(name))
        cty = ctype(dt)
        if name in written:
            sig.append(f"{cty}* __restrict__ p_{_c(name)}")
        else:
            sig.append(f"const {cty}* __restrict__ p_{_c(name)}")
        ptrs[name] = f"p_{_c(name)}"
        params.append(ParamSpec(name, "ptr", dt))
    ncell = plan.ncells
    axes = plan.axes
    rbytes = range_bytes(plan, args, scalars, dtypes, shapes)
    if rbytes is not None:
        sig += ["unsigned long long emmy_rb", "unsigned long long emmy_re"]
    use_pair = vec_ok and (pair is True or (pair == "auto" and pairable(plan, dtypes)))
    plan.pair = use_pair
    vtrip = functools.partial(_vector_trip, pair=use_pair)
    lines: list[str] = []
    w = lines.append
    w(DEVICE_PRELUDE)
    w(_VEC_HELPERS)
    lb = f"{BLOCK}, {min_blocks}" if min_blocks else f"{BLOCK}"
    w(f'extern "C" __global__ void __launch_bounds__({lb}) {kop.name}(' + ", ".join(sig) + ") {")
    w(f"    constexpr long long NCELL = {ncell}LL;")
    if rbytes is not None:
        # this launch's cells: [RB, RE)
        w("    const long long RB = (long long)(emmy_rb < (unsigned long long)NCELL ? emmy_rb : NCELL);")
        w("    const long long RE = (long long)(emmy_re < (unsigned long long)NCELL ? emmy_re : NCELL);")
    else:
        w("    constexpr long long RB = 0, RE = NCELL;")
    w("    const long long gstride = (long long)gridDim.x * blockDim.x;")
    w("    const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x;")
    scalar_env = {name: (("f32", f"p_{_c(name)}") if scalars[name] == "f32" else
                         ("int", f"(long long)p_{_c(name)}")) for name in scalars}
    if vec_ok:
        align_terms = [f"(uintptr_t)p_{_c(n)}" for n in ptrs]
        idx32 = order not in ("blocked", "tile") and ncell < (1 << 31)
        w("    const bool aligned = ((" + (" | ".join(align_terms) if align_terms else "0") + ") & 15u) == 0"
          + f" && RB % {VEC} == 0 && RE % {VEC} == 0"
          + (" && gstride <= (1LL << 27);" if idx32 else ";"))
        w("    if (aligned) {")
        ity0 = 'unsigned' if idx32 else 'long long'
        w(f"        const {ity0} NVEC = ({ity0})(RE / {VEC});  // one past this launch's last vector")
        w(f"        const {ity0} VB0 = ({ity0})(RB / {VEC});")
        if order == "tile":
            # CTA k takes TILE_U x BLOCK consecutive vectors from VB0 + k * TILE_U * BLOCK
            # (grid-stride over such tiles, so any grid is correct); every streamed load of the
            # tile is issued before any compute
            tv = tile_u * BLOCK
            # inside the loop vb < NVEC: cell offsets fit 32 bits when the problem does
            tix = ("unsigned", "u") if ncell < (1 << 31) else ("long long", "LL")

            def tile_loop(ind: str, bd: str) -> None:
                w(f"{ind}const long long tsz = {tile_u}LL * (long long)({bd});")
                w(f"{ind}for (long long vb = (long long)VB0 + (long long)blockIdx.x * tsz + threadIdx.x;"
                  " vb < (long long)NVEC; vb += (long long)gridDim.x * tsz) {")
                w(f"{ind}    const {tix[0]} vt = ({tix[0]})vb;")
                w(f"{ind}    if (vb + {tile_u - 1}LL * (long long)({bd}) < (long long)NVEC) {{")
                lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env,
                                   ["vt"] + [f"vt + {u}{tix[1]} * ({tix[0]})({bd})" for u in range(1, tile_u)],
                                   ind + "        ", ix=tix))
                w(f"{ind}    }} else {{")
                w(f"{ind}        for ({tix[0]} v = vt; v < ({tix[0]})NVEC; v += ({tix[0]})({bd})) {{")
                lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env, ["v"], ind + "            ", ix=tix))
                w(f"{ind}        }}")
                w(f"{ind}    }}")
                w(f"{ind}}}")

            # other block sizes (a foreign launch of the drop-in entry) take the scalar loop below
            w(f"        if (blockDim.x == {BLOCK}u) {{")
            tile_loop("            ", f"{BLOCK}")
            w("            return;")
            w("        }")
            w("    }")
            return _finish_vector(kop, plan, lines, ncell, unroll, vec_ok, params, why, em_path=True,
                                  shapes=shapes, dtypes=dtypes, ptrs=ptrs, scalar_env=scalar_env,
                                  rbytes=rbytes, tile_cells=tv * VEC)
        if order == "blocked":
            # CTA b owns vectors [b*per, (b+1)*per); a trip covers unroll*blockDim consecutive vectors
            w("        const long long per = ((long long)NVEC - VB0 + gridDim.x - 1) / gridDim.x;")
            w("        const long long vbeg = VB0 + (long long)blockIdx.x * per;")
            w("        const long long vend = (vbeg + per < NVEC) ? (vbeg + per) : NVEC;")
            w("        const long long bstride = blockDim.x;")
            w("        long long v = vbeg + threadIdx.x;")
            w(f"        for (; v + {unroll - 1} * bstride < vend; v += {unroll} * bstride) {{")
            lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env,
                                      ["v"] + [f"v + {u} * bstride" for u in range(1, unroll)],
                                      "            "))
            w("        }")
            w("        for (; v < vend; v += bstride) {")
            lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env, ["v"], "            "))
            w("        }")
            w("        return;")
            w("    }")
            return _finish_vector(kop, plan, lines, ncell, unroll, vec_ok, params, why, em_path=True,
                                  shapes=shapes, dtypes=dtypes, ptrs=ptrs, scalar_env=scalar_env,
                                  rbytes=rbytes)
        quantum = 1  # grid multiple that keeps hoisted broadcast operands valid
        # vector offsets in 32 bits when they stay below 2^32: c < NCELL + 4*unroll*gstride
        ity, isuf = ("unsigned", "u") if idx32 else ("long long", "LL")
        w(f"        {ity} v = VB0 + ({ity})gtid;")
        w(f"        const {ity} vgs = ({ity})gstride;")
        hoist = _hoistable(plan) if hoist_broadcast else {}
        if hoist:
            period = max(p for _, p in hoist.values())
            if period % VEC == 0:
                q = (period // VEC) // math.gcd(period // VEC, BLOCK)
                quantum = q if q <= SM_COUNT else 1
            # a thread's broadcast operands are the same on every trip when the grid
            # stride is a whole number of their periods: load them once
            w(f"        if ((gstride * {VEC}) % {period}LL == 0 && v < NVEC) {{")
            names = {}
            w(f"            const {ity} hc = v * {VEC}{isuf};")
            strides = _axis_strides(axes)
            for i, ((name, ext), st) in enumerate(zip(axes, strides)):
                q = "hc" if st == 1 else f"(hc / {st}{isuf})"
                expr = q if i == 0 else f"({q} % {ext}{isuf})"
                w(f"            const {ity} h_ax{i} = {expr};")
            for li, (ld, _) in hoist.items():
                dt = ir.canon_dtype(ld.dtype or dtypes.get(ld.input))
                pos = _axis_aligned(ld.index, axes)
                bstr = _axis_strides([axes[p_] for p_ in pos])
                off = " + ".join(f"h_ax{p_} * {bs}{isuf}" for p_, bs in zip(pos, bstr))
                var = f"hl{li}"
                if _contiguous(ld, plan):
                    w(f"            const auto {var} = emmy_ld{VEC}_{dt}({ptrs[ld.input]} + ({off}), false);")
                else:
                    w(f"            const {ctype(dt)} {var} = {ptrs[ld.input]}[{off}];")
                names[li] = var
            if pipeline:
                lines.extend(_pipelined_loop(plan, dtypes, ptrs, vtrip, shapes, scalar_env, unroll, ity, isuf,
                                             "            ", names))
            else:
                w(f"            for (; v + {unroll - 1} * vgs < NVEC; v += {unroll} * vgs) {{")
                lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env,
                                   ["v"] + [f"v + {u} * vgs" for u in range(1, unroll)],
                                   "                ", hoisted=names, ix=(ity, isuf)))
                w("            }")
            w("            for (; v < NVEC; v += vgs) {")
            lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env, ["v"], "                ",
                               hoisted=names, ix=(ity, isuf)))
            w("            }")
            w("            return;")
            w("        }")
        if pipeline and not prefetch:
            lines.extend(_pipelined_loop(plan, dtypes, ptrs, vtrip, shapes, scalar_env, unroll, ity, isuf,
                                         "        ", {}))
            w("        for (; v < NVEC; v += vgs) {")
            lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env, ["v"], "            ", ix=(ity, isuf)))
            w("        }")
            w("        return;")
            w("    }")
            return _finish_vector(kop, plan, lines, ncell, unroll, vec_ok, params, why, em_path=True,
                                  shapes=shapes, dtypes=dtypes, ptrs=ptrs, scalar_env=scalar_env,
                                  grid_quantum=quantum if vec_ok else 1, rbytes=rbytes)
        w(f"        for (; v + {unroll - 1} * vgs < NVEC; v += {unroll} * vgs) {{")
        if prefetch:
            for s_ in _streamed_loads(plan):
                for u in range(unroll):
                    w(f"            {{ const {ity} pv = v + {prefetch * unroll + u} * vgs;")
                    w(f"              if (pv < NVEC) emmy_prefetch_l2({ptrs[s_.input]} + pv * {VEC}); }}")
        lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env,
                           ["v"] + [f"v + {u} * vgs" for u in range(1, unroll)],
                           "            ", ix=(ity, isuf)))
        w("        }")
        w("        for (; v < NVEC; v += vgs) {")
        lines.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env, ["v"], "            ", ix=(ity, isuf)))
        w("        }")
        w("        return;")
        w("    }")
    return _finish_vector(kop, plan, lines, ncell, unroll, vec_ok, params, why, em_path=True,
                          shapes=shapes, dtypes=dtypes, ptrs=ptrs, scalar_env=scalar_env,
                          grid_quantum=quantum if vec_ok else 1, rbytes=rbytes)


def _pipelined_loop(plan, dtypes, ptrs, vtrip, shapes, scalar_env, unroll, ity, isuf, ind, hoisted) -> list[str]:
    """The main grid-stride loop with the streamed whole-tile loads of trip
    t+1 issued before trip t computes (register double buffer)."""
    loads = [s for s in ir.walk(plan.tile.body) if isinstance(s, ir.Load)]
    full = [li for li, s in enumerate(loads)
            if li not in hoisted and not _const_index(s.index)
            and _axis_aligned(s.index, plan.axes) == list(range(len(plan.axes)))]
    out = []
    o = out.append

    def ld(li, vexpr):
        s_ = loads[li]
        dt = ir.canon_dtype(s_.dtype or dtypes.get(s_.input))
        return f"emmy_ld{VEC}_{dt}({ptrs[s_.input]} + ({vexpr}) * {VEC}{isuf}, true)"

    for li in full:
        dt = ir.canon_dtype(loads[li].dtype or dtypes.get(loads[li].input))
        for u in range(unroll):
            o(f"{ind}EmmyVec<{ctype(dt)}, {VEC}> nx{li}_{u};")
    o(f"{ind}if (v + {unroll - 1} * vgs < NVEC) {{")
    for li in full:
        for u in range(unroll):
            o(f"{ind}    nx{li}_{u} = {ld(li, f'v + {u} * vgs')};")
    o(f"{ind}}}")
    o(f"{ind}for (; v + {unroll - 1} * vgs < NVEC; v += {unroll} * vgs) {{")
    pre = {}
    for li in full:
        for u in range(unroll):
            o(f"{ind}    const auto cu{li}_{u} = nx{li}_{u};")
            pre[(li, u)] = f"cu{li}_{u}"
    o(f"{ind}    if (v + {2 * unroll - 1} * vgs < NVEC) {{")
    for li in full:
        for u in range(unroll):
            o(f"{ind}        nx{li}_{u} = {ld(li, f'v + {unroll + u} * vgs')};")
    o(f"{ind}    }}")
    out.extend(vtrip(plan, shapes, dtypes, ptrs, scalar_env, ["v"] + [f"v + {u} * vgs" for u in range(1, unroll)],
                     ind + "    ", hoisted=hoisted, ix=(ity, isuf), preloaded=pre))
    o(f"{ind}}}")
    return out


def _finish_vector(kop, plan, lines, ncell, unroll, vec_ok, params, why, *, em_path, shapes, dtypes, ptrs,
                   scalar_env, grid_quantum: int = 1, rbytes: list[int] | None = None,
                   tile_cells: int = 0) -> KernelSource:
    """The scalar grid-stride loop (any launch, any alignment) and the launch record."""
    w = lines.append
    w("    for (long long cell = RB + gtid; cell < RE; cell += gstride) {")
    em = Emitter(shapes, dtypes, ptrs, indent="        ")
    em.env.update(scalar_env)
    _decode_axes(em, plan.axes, "cell", "ax")
    em.run(plan.tile.body)
    lines.extend(em.lines)
    w("    }")
    w("}")
    nvec = ncell // VEC if vec_ok else ncell
    per_block = BLOCK * (unroll if vec_ok else 1)
    want = (nvec + per_block - 1) // per_block
    grid = max(1, min(want, SM_COUNT * 8))
    launch = LaunchPlan(grid=(grid, 1, 1), block=(BLOCK, 1, 1), smem=0)
    if rbytes is not None:
        launch.range_total = ncell
        launch.range_align = RANGE_ALIGN
        launch.range_bytes = rbytes
    if tile_cells and rbytes is not None:
        # one CTA per tile of the launch's range (EMMY_LR_GRID_UNITS, tile_cells cells per CTA)
        launch.grid = (max(1, min(-(-ncell // tile_cells), 0x7FFFFFFF)), 1, 1)
        launch.grid_units = True
        launch.grid_quantum = tile_cells
    elif want >= SM_COUNT * 8:
        # enough work to fill the device: one wave of exactly the CTAs that fit,
        # counted by the loader for this build's registers (a partial second wave
        # of a fixed grid leaves SMs idle in a bandwidth-bound loop)
        launch.fill_waves = 1
        launch.grid_quantum = grid_quantum
    lines.append(launch_record_source("pointwise", launch, params))
    return KernelSource(entry=kop.name, source="\n".join(lines), launch=launch, params=params,
                        family="pointwise",
                        notes={"vector": vec_ok, "scalar_reasons": why, "ncells": ncell,
                               "pair": plan.pair, "order": "tile" if tile_cells else "grid"})


def _vector_trip(plan: PointwisePlan, shapes, dtypes, ptrs, scalar_env, vexprs: list[str],
                 ind: str, smem_src: dict[int, str] | None = None,
                 hoisted: dict[int, str] | None = None, pair: bool = False,
                 ix: tuple[str, str] = ("long long", "LL"),
                 preloaded: dict[tuple[int, int], str] | None = None) -> list[str]:
    """One trip: load U vectors of every input, run the cell body per lane,
    store U vectors of every output.  ``smem_src`` maps a load's position to a
    shared-memory element pointer expression (indexed by the vector's offset
    within the current tile, ``lo<u>``) for loads staged by bulk copies."""
    smem_src = smem_src or {}
    hoisted = hoisted or {}
    preloaded = preloaded or {}
    axes = plan.axes
    out: list[str] = []
    loads = [s for s in ir.walk(plan.tile.body) if isinstance(s, ir.Load)]
    writes = [s for s in ir.walk(plan.tile.body) if isinstance(s, ir.Write)]
    strides = _axis_strides(axes)
    ity, isuf = ix
    for u, vx in enumerate(vexprs):
        out.append(f"{ind}const {ity} c{u} = ({vx}) * {VEC}{isuf};")
        for i, ((name, ext), st) in enumerate(zip(axes, strides)):
            q = f"c{u}" if st == 1 else f"(c{u} / {st}{isuf})"
            expr = q if i == 0 else f"({q} % {ext}{isuf})"
            if ext == 1:
                expr = f"0{isuf}"
            out.append(f"{ind}const {ity} u{u}_ax{i} = {expr};")
    # fetch every load for every trip vector before any compute
    fetched: dict[tuple[int, int], tuple[str, bool, str]] = {}
    for li, s in enumerate(loads):
        dt = ir.canon_dtype(s.dtype or dtypes.get(s.input))
        ptr = ptrs[s.input]
        for u in range(len(vexprs)):
            var = f"ld{li}_{u}"
            if _const_index(s.index):
                off = "+".join(str(int(ix.value)) for ix in s.index) if len(s.index) == 1 else \
                    _const_flat(s, shapes)
                out.append(f"{ind}const {ctype(dt)} {var} = {ptr}[{off}];")
                fetched[(li, u)] = (var, False, dt)
                continue
            if li in smem_src:
                out.append(f"{ind}const auto {var} = emmy_lds{VEC}_{dt}({smem_src[li]} + lo{u});")
                fetched[(li, u)] = (var, True, dt)
                continue
            if li in hoisted:
                fetched[(li, u)] = (hoisted[li], _contiguous(s, plan), dt)
                continue
            if (li, u) in preloaded:
                fetched[(li, u)] = (preloaded[(li, u)], True, dt)
                continue
            pos = _axis_aligned(s.index, axes)
            bstrides = _axis_strides([axes[p] for p in pos])
            off = " + ".join(f"u{u}_ax{p} * {bs}{isuf}" for p, bs in zip(pos, bstrides)) or f"0{isuf}"
            if pos == list(range(len(axes))):
                off = f"c{u}"  # the whole tile, row-major: the cell offset itself
            contiguous = bool(pos) and pos[-1] == len(axes) - 1
            if contiguous:
                out.append(f"{ind}const auto {var} = emmy_ld{VEC}_{dt}({ptr} + ({off}), "
                           f"{'true' if _streamed(s, plan) else 'false'});")
                fetched[(li, u)] = (var, True, dt)
            else:
                out.append(f"{ind}const {ctype(dt)} {var} = {ptr}[{off}];")
                fetched[(li, u)] = (var, False, dt)
    outs: dict[tuple[int, int], list[str]] = {}
    for u in range(len(vexprs)):
        for wi, s in enumerate(writes):
            dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
            outs[(wi, u)] = [f"st{wi}_{u}_{lane}" for lane in range(VEC)]
            for lane in range(VEC):
                out.append(f"{ind}{ctype(dt)} st{wi}_{u}_{lane};")
    if pair:
        out.extend(_pair_lanes(plan, shapes, dtypes, ptrs, scalar_env, vexprs, ind, fetched, loads, writes))
    for u in range(len(vexprs) if not pair else 0):
        for lane in range(VEC):
            load_idx = {id(s): li for li, s in enumerate(loads)}
            write_idx = {id(s): wi for wi, s in enumerate(writes)}

            def load_hook(s, k, u=u, lane=lane):
                var, is_vec, dt = fetched[(load_idx[id(s)], u)]
                code = f"{var}.v[{lane}]" if is_vec else var
                return load_to_kind(code, dt)

            def write_hook(s, k, kind, code, u=u, lane=lane):
                dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
                return f"st{write_idx[id(s)]}_{u}_{lane} = {store_from(kind, code, dt)};"

            em = Emitter(shapes, dtypes, ptrs, load_hook=load_hook, write_hook=write_hook,
                         indent=ind + "    ")
            em.env.update(scalar_env)
            for i, (name, ext) in enumerate(axes):
                code = f"u{u}_ax{i}" if i < len(axes) - 1 else f"(u{u}_ax{i} + {lane})"
                em.bind_const(name, "int", code)
            em.run(plan.tile.body)
            out.append(f"{ind}{{")
            out.extend(em.lines)
            out.append(f"{ind}}}")
    for u in range(len(vexprs)):
        for wi, s in enumerate(writes):
            dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
            vals = ", ".join(outs[(wi, u)])
            out.append(f"{ind}emmy_st{VEC}_{dt}({ptrs[s.output]} + c{u}, {vals});")
    return out


def _pair_lanes(plan, shapes, dtypes, ptrs, scalar_env, vexprs, ind, fetched, loads, writes) -> list[str]:
    """The cell body once per pair of adjacent lanes (0,1), (2,3) of each trip
    vector, every f32 value an ``EmmyF2``."""
    out: list[str] = []
    load_idx = {id(s): li for li, s in enumerate(loads)}
    write_idx = {id(s): wi for wi, s in enumerate(writes)}
    for u in range(len(vexprs)):
        for l0 in range(0, VEC, 2):
            l1 = l0 + 1

            def load_hook(s, k, u=u, l0=l0, l1=l1):
                var, is_vec, dt = fetched[(load_idx[id(s)], u)]
                if not is_vec:
                    return "f32", f"EmmyF2({load_to_kind(var, dt)[1]})"
                a = load_to_kind(f"{var}.v[{l0}]", dt)[1]
                b = load_to_kind(f"{var}.v[{l1}]", dt)[1]
                return "f32", f"EmmyF2(make_float2({a}, {b}))"

            def write_hook(s, k, kind, code, u=u, l0=l0, l1=l1):
                dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
                wi = write_idx[id(s)]
                return (f"{{ const EmmyF2 w_ = {code}; st{wi}_{u}_{l0} = {store_from('f32', 'w_.v.x', dt)}; "
                        f"st{wi}_{u}_{l1} = {store_from('f32', 'w_.v.y', dt)}; }}")

            em = Emitter(shapes, dtypes, ptrs, load_hook=load_hook, write_hook=write_hook,
                         indent=ind + "    ")
            em.ftype = "EmmyF2"
            em.env.update(scalar_env)
            em.run(plan.tile.body)
            out.append(f"{ind}{{")
            out.extend(em.lines)
            out.append(f"{ind}}}")
    return out


RANGE_ALIGN = 4096  # cells: range ends keep vectors, hoisting periods up to 16 KB and pages whole


def range_bytes(plan: PointwisePlan, args: list[str], scalars: dict, dtypes: dict,
                shapes: dict) -> list[int] | None:
    """Bytes per cell of each parameter for ranged launches (cell c of a
    whole-tile buffer is element c), 0 for parameters read whole; None when
    some output is written other than element-per-cell, so a range of cells
    would write bytes outside its range."""
    axes = plan.axes
    full: dict[str, bool] = {}
    written: set[str] = set()
    for s in ir.walk(plan.tile.body):
        if isinstance(s, (ir.Load, ir.Write)):
            buf = s.input if isinstance(s, ir.Load) else s.output
            pos = _axis_aligned(s.index, axes)
            shape = [int(d) for d in shapes.get(buf, ())]
            ok = (pos == list(range(len(axes))) and shape == [ext for _, ext in axes]
                  and (isinstance(s, ir.Load) or len(s.values) == 1))
            full[buf] = full.get(buf, True) and ok
            if isinstance(s, ir.Write):
                written.add(buf)
                if not ok or s.atomic:
                    return None
    out = []
    for name in args:
        if name in scalars or name not in full or not full[name]:
            out.append(0)
            continue
        out.append(ELEM_BYTES.get(ir.canon_dtype(dtypes.get(name)), 4))
    return out


PAIR_OPS = {"add", "sum", "subtract", "sub", "multiply", "mul", "divide", "true_divide", "div",
            "maximum", "amax", "max", "minimum", "amin", "min", "exp2", "exp", "exp_fast", "sqrt",
            "rsqrt", "reciprocal", "recip", "square", "clamp", "clip", "relu", "leaky_relu", "neg",
            "negative", "abs", "absolute", "copy", "log", "log_fast", "log2", "lg2", "tanh",
            "sigmoid", "silu", "pow"}


def pairable(plan: PointwisePlan, dtypes: dict) -> bool:
    """True when the cell body is straight-line f32 arithmetic that reads no
    axis value: loads, float literals, ops of ``PAIR_OPS`` and plain writes.
    Such a body computes two adjacent cells independently in the two lanes
    of an ``EmmyF2`` with the same per-lane rounding."""
    axis_names = {a for a, _ in plan.axes}
    for s in ir.walk(plan.tile.body):
        if isinstance(s, ir.Load):
            if ir.canon_dtype(s.dtype or dtypes.get(s.input)) not in ("f32", "bf16", "f16"):
                return False
        elif isinstance(s, ir.Write):
            if s.atomic or ir.canon_dtype(s.value_dtype or dtypes.get(s.output)) not in ("f32", "bf16", "f16"):
                return False
            if any(not isinstance(v, str) for v in s.values):
                return False
        elif isinstance(s, ir.Let):
            if not (isinstance(s.value, ir.Literal) and isinstance(s.value.value, float)):
                return False
        elif isinstance(s, ir.Assign):
            if ir.op_name(s.op) not in PAIR_OPS:
                return False
            if s.dtype is not None and ir.canon_dtype(s.dtype) != "f32":
                return False
            if any(isinstance(a, str) and a in axis_names for a in s.args):
                return False
            if any(not isinstance(a, str) for a in s.args):
                return False
        else:
            return False
    return True


def _contiguous(s: ir.Load, plan: PointwisePlan) -> bool:
    pos = _axis_aligned(s.index, plan.axes)
    return bool(pos) and pos[-1] == len(plan.axes) - 1


def _hoistable(plan: PointwisePlan) -> dict[int, tuple[ir.Load, int]]:
    """Broadcast loads indexed by a proper suffix of the tile axes: their value
    for cell c depends only on c mod P (P = product of those axes' extents).
    Maps load position -> (load, P)."""
    out = {}
    loads = [t for t in ir.walk(plan.tile.body) if isinstance(t, ir.Load)]
    n = len(plan.axes)
    for li, ld in enumerate(loads):
        if _const_index(ld.index) or _streamed(ld, plan):
            continue
        pos = _axis_aligned(ld.index, plan.axes)
        if not pos or pos != list(range(pos[0], n)):
            continue
        period = 1
        for p_ in pos:
            period *= plan.axes[p_][1]
        out[li] = (ld, period)
    return out


def _const_flat(s: ir.Load, shapes) -> str:
    shape = shapes.get(s.input)
    vals = [int(ix.value) for ix in s.index]
    if not shape or len(shape) != len(vals):
        return str(sum(vals))
    acc = 0
    for v, st in zip(vals, _axis_strides([(None, int(e)) for e in shape])):
        acc += v * st
    return str(acc)


def _streamed(s: ir.Load, plan: PointwisePlan) -> bool:
    """Full-tile operands are read once: stream them past L1/L2 residency."""
    pos = _axis_aligned(s.index, plan.axes)
    return pos is not None and len(pos) == len(plan.axes)


_VEC_HELPERS = r"""
template <class T, int N> struct EmmyVec { T v[N]; };
static __device__ __forceinline__ void emmy_prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" :: "l"(p));
}
static __device__ __forceinline__ EmmyVec<float, 4> emmy_lds4_f32(const float* p) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    return EmmyVec<float, 4>{{t.x, t.y, t.z, t.w}};
}
static __device__ __forceinline__ EmmyVec<__nv_bfloat16, 4> emmy_lds4_bf16(const __nv_bfloat16* p) {
    EmmyVec<__nv_bfloat16, 4> r;
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    memcpy(&r, &t, 8);
    return r;
}
static __device__ __forceinline__ EmmyVec<__half, 4> emmy_lds4_f16(const __half* p) {
    EmmyVec<__half, 4> r;
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    memcpy(&r, &t, 8);
    return r;
}
static __device__ __forceinline__ EmmyVec<float, 4> emmy_ld4_f32(const float* p, bool stream) {
    float4 t = stream ? __ldcs(reinterpret_cast<const float4*>(p))
                      : __ldg(reinterpret_cast<const float4*>(p));
    return EmmyVec<float, 4>{{t.x, t.y, t.z, t.w}};
}
static __device__ __forceinline__ void emmy_st4_f32(float* p, float a, float b, float c, float d) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(a, b, c, d));
}
static __device__ __forceinline__ EmmyVec<__nv_bfloat16, 4> emmy_ld4_bf16(const __nv_bfloat16* p, bool stream) {
    uint2 t = stream ? __ldcs(reinterpret_cast<const uint2*>(p)) : __ldg(reinterpret_cast<const uint2*>(p));
    EmmyVec<__nv_bfloat16, 4> r;
    memcpy(&r, &t, 8);
    return r;
}
static __device__ __forceinline__ void emmy_st4_bf16(__nv_bfloat16* p, __nv_bfloat16 a, __nv_bfloat16 b,
                                                     __nv_bfloat16 c, __nv_bfloat16 d) {
    EmmyVec<__nv_bfloat16, 4> r{{a, b, c, d}};
    uint2 t; memcpy(&t, &r, 8);
    __stcs(reinterpret_cast<uint2*>(p), t);
}
static __device__ __forceinline__ EmmyVec<__half, 4> emmy_ld4_f16(const __half* p, bool stream) {
    uint2 t = stream ? __ldcs(reinterpret_cast<const uint2*>(p)) : __ldg(reinterpret_cast<const uint2*>(p));
    EmmyVec<__half, 4> r;
    memcpy(&r, &t, 8);
    return r;
}
static __device__ __forceinline__ void emmy_st4_f16(__half* p, __half a, __half b, __half c, __half d) {
    EmmyVec<__half, 4> r{{a, b, c, d}};
    uint2 t; memcpy(&t, &r, 8);
    __stcs(reinterpret_cast<uint2*>(p), t);
}
"""


def _generate_bulk(kop, plan: PointwisePlan, shapes, dtypes, args, scalars, written,
                   streamed: list[ir.Load]) -> KernelSource:
    """Large vectorisable tiles: a producer warp streams each full-tile input
    through a shared-memory ring with 1-D bulk async copies (``cp.async.bulk``,
    completion on an mbarrier), so tens of KB per SM are in flight without
    costing registers; 8 consumer warps run the cell body from shared memory
    and store 128-bit vectors straight to global memory.  Misaligned pointers
    fall back to the register-vector loop."""
    from ..cgen import DEVICE_PRELUDE as _P  # noqa: F401  (same prelude as the other paths)
    params: list[ParamSpec] = []
    ptrs: dict[str, str] = {}
    sig: list[str] = []
    for name in args:
        if name in scalars:
            dt = scalars[name]
            sig.append(f"{ctype(dt)} p_{_c(name)}")
            params.append(ParamSpec(name, "scalar", dt))
            continue
        dt = ir.canon_dtype(dtypes.get(name))
        cty = ctype(dt)
        sig.append(f"{cty}* __restrict__ p_{_c(name)}" if name in written
                   else f"const {cty}* __restrict__ p_{_c(name)}")
        ptrs[name] = f"p_{_c(name)}"
        params.append(ParamSpec(name, "ptr", dt))
    scalar_env = {name: (("f32", f"p_{_c(name)}") if scalars[name] == "f32" else
                         ("int", f"(long long)p_{_c(name)}")) for name in scalars}
    loads = [s for s in ir.walk(plan.tile.body) if isinstance(s, ir.Load)]
    inputs = []          # unique streamed buffers, in first-use order
    for s in streamed:
        if s.input not in inputs:
            inputs.append(s.input)
    esz = {n: ir.ELEM_BYTES[ir.canon_dtype(dtypes.get(n))] for n in inputs}
    offs, off = {}, 0
    for n in inputs:
        offs[n] = off
        off += -(-BULK_TILE * esz[n] // 128) * 128
    stage_bytes = off
    stages = max(2, min(4, BULK_SMEM_TARGET // stage_bytes))
    smem = stages * stage_bytes + 2 * stages * 8 + 16
    ncell = plan.ncells
    tiles = -(-ncell // BULK_TILE)
    smem_src = {}
    for li, s in enumerate(loads):
        if s in streamed:
            dt = ir.canon_dtype(s.dtype or dtypes.get(s.input))
            smem_src[li] = (f"reinterpret_cast<const {ctype(dt)}*>(stage_base + {offs[s.input]}u)")
    L: list[str] = []
    w = L.append
    w(DEVICE_PRELUDE)
    w(_VEC_HELPERS)
    w('#include "emmy_sm100.cuh"')
    nthreads = BULK_CONSUMERS + 32
    w(f'extern "C" __global__ void __launch_bounds__({nthreads}, {BULK_CTAS_PER_SM}) {kop.name}(' + ", ".join(sig) + ") {")
    w(f"    constexpr long long NCELL = {ncell}LL, NVEC = NCELL / {VEC}, TILES = {tiles}LL;")
    w(f"    constexpr int TILE = {BULK_TILE}, STAGES = {stages}, CONS = {BULK_CONSUMERS};")
    w(f"    constexpr uint32_t STAGE_BYTES = {stage_bytes}u, SMEM_BYTES = {smem}u;")
    w("    constexpr uint64_t WAIT_NS = 2000000000ull;")
    align_terms = [f"(uintptr_t){p}" for p in ptrs.values()]
    w("    uint32_t dyn_smem;")
    w('    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));')
    w("    const bool aligned = ((" + (" | ".join(align_terms) or "0") + ") & 15u) == 0;")
    w(f"    if (blockDim.x != {nthreads} || blockDim.y != 1 || blockDim.z != 1 || dyn_smem < SMEM_BYTES || !aligned) {{")
    w("        // any other launch or misaligned buffers: register-vector / scalar grid-stride loops")
    w("        const long long gstride = (long long)gridDim.x * blockDim.x * blockDim.y * blockDim.z;")
    w("        const long long gtid = (long long)blockIdx.x * blockDim.x * blockDim.y * blockDim.z"
      " + (threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x;")
    w("        if (aligned) {")
    w("            for (long long v = gtid; v < NVEC; v += gstride) {")
    L.extend(_vector_trip(plan, shapes, dtypes, ptrs, scalar_env, ["v"], "                "))
    w("            }")
    w("            return;")
    w("        }")
    w("        for (long long cell = gtid; cell < NCELL; cell += gstride) {")
    em = Emitter(shapes, dtypes, ptrs, indent="            ")
    em.env.update(scalar_env)
    _decode_axes(em, plan.axes, "cell", "ax")
    em.run(plan.tile.body)
    L.extend(em.lines)
    w("        }")
    w("        return;")
    w("    }")
    w("    extern __shared__ __align__(128) uint8_t smem[];")
    w("    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);")
    w("    uint64_t *empty = full + STAGES;")
    w("    volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(empty + STAGES);")
    w("    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;")
    w("    if (threadIdx.x == 0) {")
    w("        for (int s = 0; s < STAGES; ++s) { emmy::mbar_init(&full[s], 1); emmy::mbar_init(&empty[s], CONS / 32); }")
    w("        *abort_flag = 0u;")
    w("        emmy::fence_barrier_init();")
    w("    }")
    w("    __syncthreads();")
    w("    if (warp == CONS / 32) {")
    w("        if (lane == 0) {")
    w("            // producer: bulk-copy each tile of every streamed input into the ring")
    w("            uint32_t issued = 0u, parity_bits = 0u;")
    w("            bool ok = true;")
    w("            int j = 0;")
    w("            for (long long t = blockIdx.x; t < TILES; t += gridDim.x, ++j) {")
    w("                const int s = j % STAGES;")
    w("                const uint32_t ph = (uint32_t)(j / STAGES) & 1u;")
    w("                if (!emmy::mbar_wait(&empty[s], ph ^ 1u, abort_flag, EMMY_STATUS_TIMEOUT_PRODUCER, WAIT_NS)) { ok = false; break; }")
    w("                const long long base = t * TILE;")
    w("                const uint32_t cnt = (uint32_t)((NCELL - base) < TILE ? (NCELL - base) : TILE);")
    total = " + ".join(f"cnt * {esz[n]}u" for n in inputs)
    w(f"                emmy::mbar_arrive_expect_tx(&full[s], {total});")
    for n in inputs:
        w(f"                emmy::bulk_load(smem + s * STAGE_BYTES + {offs[n]}u, {ptrs[n]} + base, cnt * {esz[n]}u, &full[s]);")
    w("                issued |= 1u << s;")
    w("                parity_bits = (parity_bits & ~(1u << s)) | (ph << s);")
    w("            }")
    w("            if (!ok) {")
    w("                volatile uint32_t never = 0u;")
    w("                for (int s = 0; s < STAGES; ++s)")
    w("                    if (issued & (1u << s)) emmy::mbar_wait(&full[s], (parity_bits >> s) & 1u, &never, 0u, 20000000ull);")
    w("            }")
    w("        }")
    w("        __syncwarp();")
    w("    } else {")
    w("        // consumers: 4 vectors of 4 cells per thread per tile, straight from shared memory")
    w("        int j = 0;")
    w("        for (long long t = blockIdx.x; t < TILES; t += gridDim.x, ++j) {")
    w("            const int s = j % STAGES;")
    w("            const uint32_t ph = (uint32_t)(j / STAGES) & 1u;")
    w("            if (!emmy::mbar_wait(&full[s], ph, abort_flag, EMMY_STATUS_TIMEOUT_EPILOGUE, WAIT_NS)) break;")
    w("            const uint8_t *stage_base = smem + s * STAGE_BYTES;")
    w("            const long long vb = t * (TILE / 4);")
    for u in range(4):
        w(f"            if (vb + {u} * CONS + tid < NVEC) {{")
        w(f"                const int lo0 = ({u} * CONS + tid) * 4;")
        L.extend(_vector_trip(plan, shapes, dtypes, ptrs, scalar_env, [f"vb + {u} * CONS + tid"],
                              "                ", smem_src))
        w("            }")
    w("            __syncwarp();")
    w("            if (lane == 0) emmy::mbar_arrive(&empty[s]);")
    w("        }")
    w("    }")
    w("}")
    grid = max(1, min(tiles, SM_COUNT * BULK_CTAS_PER_SM))
    launch = LaunchPlan(grid=(grid, 1, 1), block=(nthreads, 1, 1), smem=smem)
    L.append(launch_record_source("pointwise", launch, params))
    return KernelSource(entry=kop.name, source="\n".join(L), launch=launch, params=params,
                        family="pointwise",
                        notes={"vector": True, "bulk": True, "stages": stages, "tile": BULK_TILE,
                               "scalar_reasons": [], "ncells": ncell})
