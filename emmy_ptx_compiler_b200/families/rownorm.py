"""Row-fused family: reductions over a row followed by a pointwise pass over
the same row, in one kernel (rmsnorm, softmax, l2norm and the like).

Recognises the reference's block-per-row schedule with several passes
(compile.py:1866-1914 for each ``StridedLoop``, 2201-2286 for the
``WarpShuffle``/``TreeHalve`` combine after each reducing pass; the f01-f03
fused kernels of tools/make_proxy_set.py:393-414): a Tile over
``(rows..., co)`` whose body is a sequence of

* reducing passes ``StridedLoop(k, start=co, step=|co|)`` with ``Accum``s,
  each followed by its warp/tree combine, after which every thread holds the
  row's result (TreeHalve re-reads the root slot, compile.py:2271-2277);
* per-row scalar statements (``Let``/``Assign``/``Init``, leader writes under
  ``co == 0``);
* mapping passes ``StridedLoop(k, ...)`` without ``Accum`` that write
  ``out[row..., k]``.

The reference rereads the row from global memory in every pass.  Here rows
of at least ``ROW_PER_CTA_BYTES`` get one CTA each, rows whose values fit one
warp's registers get one warp each (``WR_ROWS`` rows per CTA, reductions
within the warp), and the launch's grid follows its row range in both cases;
other rows run on a persistent grid sized by the loader from occupancy, one
CTA per row at a time.  The row is read once with 128-bit loads into registers when it
fits (up to 64 floats per thread), every pass runs on those registers, each
reduction is a ``__shfl_xor_sync`` butterfly plus one shared-memory stage
that every thread combines in the same fixed warp order, and the output is
written once with streaming 128-bit stores.  HBM traffic is one read of the
row and one write, against two or three reads plus a write in the
reference.  Rows longer than the register budget reread the row from L2 per
pass.  Reductions sum in a different order than the reference (rtol bar);
element arithmetic is the reference's op table, FMA contraction included.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .. import ir
from ..cgen import (DEVICE_PRELUDE, DIVIDE_OPS, Emitter, combine_code, ctype, f32_lit, fusable_products, identity_of,
                    lit_int, load_to_kind, store_from)
from ..errors import UnsupportedIR
from .common import KernelSource, LaunchPlan, ParamSpec, SM_COUNT, launch_record_source
from .common import c_ident as _c
from .pointwise import _VEC_HELPERS

MAX_THREADS = 256
CACHE_FLOATS = 64          # per thread: rows whose streamed tensors fit stay in registers
# a streamed row this long gets a CTA of its own: CTAs that end after one row let the
# SM start the next row's loads while the last row's stores drain (16384 x 8192 f32:
# 0.159 ms against 0.178 ms for a persistent grid of 4 CTAs per SM)
ROW_PER_CTA_BYTES = 16 * 1024
# shorter rows whose streamed values fit one warp's registers run one row per warp, this many
# rows per CTA: reductions are butterflies within the warp, and no CTA barrier is taken
WR_ROWS = 8
_SCHEDULE = (ir.WarpShuffle, ir.TreeHalve, ir.Smem, ir.Sync)
_PASS_STMTS = (ir.Load, ir.Let, ir.Init, ir.Assign, ir.Accum, ir.Write, ir.Select, ir.Cond)
_COMBINE = {"add": "add", "sum": "add", "maximum": "maximum", "amax": "maximum", "max": "maximum",
            "minimum": "minimum", "amin": "minimum", "min": "minimum", "multiply": "multiply",
            "prod": "multiply"}


@dataclass
class Pass:
    loop: ir.StridedLoop
    accs: list[tuple[str, str]]            # (name, combine op); empty for a mapping pass


@dataclass
class RowPlan:
    tile: ir.Tile
    row_axes: list[tuple[str, int]]
    co: str
    K: int
    steps: list                            # Pass | ("row", stmt) | ("leader", stmt)
    streamed: list[str]                    # tensors read as [rows..., K]
    vectors: list[str]                     # tensors read as [K]
    outputs: list[str]                     # tensors written as [rows..., K]
    notes: dict = field(default_factory=dict)

    @property
    def rows(self) -> int:
        n = 1
        for _, e in self.row_axes:
            n *= e
        return n


def _unwrap_leader(s, co: str):
    if isinstance(s, ir.Cond) and not s.else_body and isinstance(s.cond, ir.BinaryExpr):
        c = s.cond
        if c.op == "==" and isinstance(c.left, ir.Var) and c.left.name == co and lit_int(c.right) == 0:
            return s.body
    return None


def _smem_cond(s, smem: set[str]) -> bool:
    if not isinstance(s, ir.Cond):
        return False
    inner = list(ir.walk(s.body)) + list(ir.walk(s.else_body))
    return bool(inner) and all(isinstance(t, ir.Write) and t.output in smem for t in inner)


def _index_names(index) -> list[str] | None:
    out = []
    for ix in index:
        if not isinstance(ix, ir.Var):
            return None
        out.append(ix.name)
    return out


def _defines(s) -> list[str]:
    if isinstance(s, ir.Load):
        return list(s.names)
    if isinstance(s, (ir.Assign, ir.Let, ir.Init, ir.Select, ir.Accum)):
        return [s.name]
    return []


def match(kop: ir.KernelOp, shapes: dict, dtypes: dict) -> RowPlan | None:
    body = ir.body_stmts(kop.body)
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        return None
    tile = body[0]
    stmts = list(ir.body_stmts(tile.body))
    axes = [(a.name, a.size) for a in tile.axes]
    loops = [s for s in stmts if isinstance(s, ir.StridedLoop)]
    if len(axes) < 2 or not loops:
        return None
    if any(isinstance(s, ir.Loop) for s in stmts):
        return None
    co, co_ext = axes[-1]
    row_axes = axes[:-1]
    row_names = [a for a, _ in row_axes]
    K = None
    for lp in loops:
        if not (isinstance(lp.start, ir.Var) and lp.start.name == co and lit_int(lp.step) == co_ext):
            return None
        end = lp.axis.size if lp.end is None else lit_int(lp.end)
        if end is None or end != lp.axis.size:
            return None
        if K is None:
            K = end
        elif K != end:
            return None
        if not all(isinstance(t, _PASS_STMTS) for t in ir.walk(lp.body)):
            return None
    smem = {s.name for s in ir.walk(tile.body) if isinstance(s, ir.Smem)}
    # names defined nowhere in the kernel are its scalar parameters (or builtins)
    defined_anywhere = set(smem) | {a for a, _ in axes} | {lp.axis.name for lp in loops}
    for t in ir.walk(tile.body):
        defined_anywhere |= set(_defines(t))
        if isinstance(t, (ir.WarpShuffle, ir.TreeHalve)):
            defined_anywhere |= set(t.state_b)
    steps: list = []
    streamed, vectors, outputs = [], [], []
    row_defined: set[str] = set(row_names)
    pending: set[str] = set()               # accumulators awaiting their TreeHalve
    for s in stmts:
        if isinstance(s, ir.TreeHalve):
            pending -= set(s.state)
            continue
        if isinstance(s, _SCHEDULE) or _smem_cond(s, smem):
            continue
        lead = _unwrap_leader(s, co)
        if isinstance(s, ir.StridedLoop):
            if pending:
                return None
            accs: list[tuple[str, str]] = []
            local: set[str] = {s.axis.name}
            for t in ir.walk(s.body):
                if isinstance(t, ir.Accum):
                    if t.base not in (None, t.name):
                        return None
                    op = _COMBINE.get(ir.op_name(t.op))
                    if op is None:
                        return None
                    if isinstance(t, ir.Accum) and t.name not in [a for a, _ in accs]:
                        accs.append((t.name, op))
                if isinstance(t, (ir.Cond, ir.Select)):
                    if any(isinstance(u, (ir.Accum, ir.Write)) for u in ir.walk(getattr(t, "body", ()))):
                        return None
                for n in t.reads():
                    if n in row_defined or n in local or n == s.axis.name or n not in defined_anywhere:
                        continue
                    if isinstance(t, ir.Accum) and n == t.name:
                        continue
                    return None                      # reads the co lane or a name it does not see
                if isinstance(t, ir.Load):
                    nm = _index_names(t.index)
                    shp = [int(d) for d in shapes.get(t.input, ())]
                    if nm == row_names + [s.axis.name] and shp == [e for _, e in row_axes] + [K]:
                        if t.input not in streamed:
                            streamed.append(t.input)
                    elif nm == [s.axis.name] and shp == [K]:
                        if t.input not in vectors:
                            vectors.append(t.input)
                    elif t.index and any(n == s.axis.name for n in (nm or [])):
                        return None
                if isinstance(t, ir.Write):
                    nm = _index_names(t.index)
                    shp = [int(d) for d in shapes.get(t.output, ())]
                    if t.atomic or len(t.values) != 1 or nm != row_names + [s.axis.name] \
                            or shp != [e for _, e in row_axes] + [K]:
                        return None
                    if t.output not in outputs:
                        outputs.append(t.output)
                local |= set(_defines(t))
            if accs and any(isinstance(t, ir.Write) for t in ir.walk(s.body)):
                return None
            steps.append(Pass(s, accs))
            pending |= {a for a, _ in accs}
            row_defined |= {a for a, _ in accs}
            continue
        inner = lead if lead is not None else (s,)
        for t in ir.walk(inner):
            if not isinstance(t, (ir.Let, ir.Assign, ir.Init, ir.Write, ir.Load, ir.Cond, ir.Select)):
                return None
            if pending and (set(t.reads()) & pending):
                return None                      # reads a partial accumulator
            if co in t.reads():
                return None
            if isinstance(t, ir.Write) and t.atomic:
                return None
        steps.append(("leader" if lead is not None else "row", s if lead is None else tuple(lead)))
        for t in ir.walk(inner):
            row_defined |= set(_defines(t))
    if pending or not outputs:
        return None
    if not any(isinstance(p, Pass) and p.accs for p in steps):
        return None
    for name in streamed + vectors + outputs:
        if ir.canon_dtype(dtypes.get(name)) not in ("f32", "bf16", "f16"):
            raise UnsupportedIR(f"row-fused kernel on {dtypes.get(name)} tensor {name!r}")
    return RowPlan(tile, row_axes, co, K, steps, streamed, vectors, outputs)


def range_bytes(plan: RowPlan, args: list[str], scalars: dict, dtypes: dict, shapes: dict) -> list[int]:
    """Bytes per row of each parameter for row-range launches: a row of the
    streamed inputs and outputs, one element of [rows...]-shaped buffers,
    0 (read whole) for the rest."""
    rows_shape = [e for _, e in plan.row_axes]
    out = []
    for name in args:
        if name in scalars:
            out.append(0)
            continue
        esz = ir.ELEM_BYTES.get(ir.canon_dtype(dtypes.get(name)), 4)
        shp = [int(d) for d in shapes.get(name, ())]
        if name in plan.streamed or name in plan.outputs:
            out.append(plan.K * esz)
        elif shp == rows_shape and shp:
            out.append(esz)
        else:
            out.append(0)
    return out


def generate(kop: ir.KernelOp, plan: RowPlan, shapes: dict, dtypes: dict, args: list[str],
             scalars: dict[str, str], written: set[str], *, bulk_prefetch: bool = False,
             reuse_values: bool = True, warp_rows: bool = True) -> KernelSource:
    """``warp_rows``: rows short enough for one warp's registers run one row per
    warp, ``WR_ROWS`` rows per CTA (reductions are warp butterflies, no CTA
    barrier); longer rows run one row per CTA of up to ``MAX_THREADS``."""
    params: list[ParamSpec] = []
    ptrs: dict[str, str] = {}
    sig: list[str] = []
    for name in args:
        if name in scalars:
            sig.append(f"{ctype(scalars[name])} p_{_c(name)}")
            params.append(ParamSpec(name, "scalar", scalars[name]))
            continue
        dt = ir.canon_dtype(dtypes.get(name))
        const = "" if name in written else "const "
        sig.append(f"{const}{ctype(dt)}* __restrict__ p_{_c(name)}")
        ptrs[name] = f"p_{_c(name)}"
        params.append(ParamSpec(name, "ptr", dt))
    sig += ["unsigned long long emmy_rb", "unsigned long long emmy_re"]
    scalar_env = {n: (("f32", f"p_{_c(n)}") if scalars[n] == "f32" else ("int", f"(long long)p_{_c(n)}"))
                  for n in scalars}
    K = plan.K
    vec = K % 4 == 0
    nred = sum(len(p.accs) for p in plan.steps if isinstance(p, Pass))
    fus = fusable_products(plan.tile.body)

    def threads_for(vw: int) -> int:
        units = -(-K // vw)
        return max(32, min(MAX_THREADS, -(-units // 32) * 32))

    T = threads_for(4 if vec else 1)
    nvec4 = -(-K // 4)
    row_bytes = K * max([ir.ELEM_BYTES[ir.canon_dtype(dtypes.get(n))] for n in plan.streamed] or [0])
    wr = (warp_rows and vec and not bulk_prefetch and plan.rows >= WR_ROWS and row_bytes < ROW_PER_CTA_BYTES
          and -(-nvec4 // 32) * 4 * max(1, len(plan.streamed)) <= CACHE_FLOATS)
    if wr:
        T = 32                     # threads per row; the CTA holds WR_ROWS rows
    CT = T * WR_ROWS if wr else T  # threads per CTA
    NW = T // 32
    lines: list[str] = []
    w = lines.append
    w(DEVICE_PRELUDE)
    w(_VEC_HELPERS)
    w('#include "emmy_sm100.cuh"')
    w(f'extern "C" __global__ void __launch_bounds__({CT}) {kop.name}(' + ", ".join(sig) + ") {")
    w(f"    constexpr long long NROWS = {plan.rows}LL, K = {K}LL;")
    if not wr:
        w(f"    __shared__ float red_smem[{max(1, nred)}][{NW}];")
    w(f"    if (blockDim.x != {CT} || blockDim.y != 1 || blockDim.z != 1) {{")
    w("        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);")
    w("        return;")
    w("    }")
    w("    const long long RB = (long long)(emmy_rb < (unsigned long long)NROWS ? emmy_rb : NROWS);")
    w("    const long long RE = (long long)(emmy_re < (unsigned long long)NROWS ? emmy_re : NROWS);")
    if wr:
        # one warp per row: tid is the lane, wrow the warp's row slot in the CTA
        w("    const int tid = threadIdx.x & 31, lane = tid, wrow = threadIdx.x >> 5;")
    else:
        w("    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;")
    cached4 = -(-nvec4 // T) * 4 * max(1, len(plan.streamed)) <= CACHE_FLOATS
    stage = _stage_bytes(plan, dtypes)
    bulk = bulk_prefetch and vec and cached4 and bool(plan.streamed) and stage <= STAGE_BYTES_MAX
    dyn = 0
    if bulk:
        # dynamic shared memory: one stage per streamed tensor, then the mbarrier and flags
        offs = {}
        cur = 0
        for n in plan.streamed:
            offs[n] = cur
            cur += K * ir.ELEM_BYTES[ir.canon_dtype(dtypes.get(n))]
        bar_off = (cur + 15) // 16 * 16
        dyn = bar_off + 16
        w("    extern __shared__ __align__(16) unsigned char rn_smem[];")
        for n in plan.streamed:
            dt = ir.canon_dtype(dtypes.get(n))
            w(f"    {ctype(dt)} *const stage_{_c(n)} = reinterpret_cast<{ctype(dt)} *>(rn_smem + {offs[n]});")
        w(f"    uint64_t *const rn_bar = reinterpret_cast<uint64_t *>(rn_smem + {bar_off});")
        w(f"    volatile uint32_t *const rn_abort = reinterpret_cast<volatile uint32_t *>(rn_smem + {bar_off + 8});")
        w("    uint32_t rn_dyn;")
        w('    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(rn_dyn));')
    if vec:
        terms = [f"(uintptr_t){ptrs[n]}" for n in plan.streamed + plan.vectors + plan.outputs]
        w("    const bool aligned = ((" + " | ".join(terms) + ") & 15u) == 0;")
        if bulk:
            w(f"    if (aligned && rn_dyn >= {dyn}u) {{")
            w("        if (tid == 0) {")
            w("            emmy::mbar_init(rn_bar, 1);")
            w("            *rn_abort = 0u;")
            w("            emmy::fence_barrier_init();")
            w("        }")
            w("        __syncthreads();")
            lines.extend(_row_loop(plan, shapes, dtypes, ptrs, scalar_env, fus, 4, T, "        ", bulk=True,
                                   reuse_values=reuse_values))
            w("    } else if (aligned) {")
        else:
            w("    if (aligned) {")
        lines.extend(_row_loop(plan, shapes, dtypes, ptrs, scalar_env, fus, 4, T, "        ",
                               reuse_values=reuse_values, wr=wr))
        w("    } else {")
        lines.extend(_row_loop(plan, shapes, dtypes, ptrs, scalar_env, fus, 1, T, "        ",
                               reuse_values=reuse_values, wr=wr))
        w("    }")
    else:
        lines.extend(_row_loop(plan, shapes, dtypes, ptrs, scalar_env, fus, 1, T, "    ",
                               reuse_values=reuse_values))
    w("}")
    per_row = vec and row_bytes >= ROW_PER_CTA_BYTES
    # warps whose row fills their registers (16 float4 per lane) take two rows each: measured
    # 6.6 against 6.2 TB/s at 65536 x 2048 (rmsnorm, 154 registers, one CTA per SM)
    wr_rounds = 2 if wr and -(-nvec4 // 32) >= 16 else 1
    if wr:
        grid = max(1, min(-(-plan.rows // (WR_ROWS * wr_rounds)), 0x7FFFFFFF))
    else:
        grid = max(1, min(plan.rows, 0x7FFFFFFF if per_row else SM_COUNT * 8))
    launch = LaunchPlan(grid=(grid, 1, 1), block=(CT, 1, 1), smem=dyn, range_total=plan.rows, range_align=1,
                        range_bytes=range_bytes(plan, args, scalars, dtypes, shapes), grid_units=per_row or wr)
    if wr:
        launch.grid_quantum = WR_ROWS * wr_rounds   # units (rows) per CTA for the range-sized grid
    if plan.rows >= SM_COUNT * 8 and not per_row and not wr:
        launch.fill_waves = 1
    lines.append(launch_record_source("rownorm", launch, params))
    nvec = -(-K // 4) if vec else K
    ept = -(-nvec // T)
    notes = {"kernel": "row_fused", "threads": CT, "threads_per_row": T,
             "rows_per_cta": WR_ROWS * wr_rounds if wr else 1,
             "vector": vec, "passes": sum(isinstance(p, Pass) for p in plan.steps),
             "reductions": nred, "elems_per_thread": ept * (4 if vec else 1),
             "cached": ept * (4 if vec else 1) * max(1, len(plan.streamed)) <= CACHE_FLOATS,
             "bulk_prefetch": bool(bulk), "cta_per_row": per_row, "warp_per_row": wr}
    return KernelSource(entry=kop.name, source="\n".join(lines), launch=launch, params=params, family="rownorm",
                        notes=notes)


STAGE_BYTES_MAX = 96 * 1024   # shared-memory stage for the next row (bulk prefetch)
KEEP_MAX = 2                  # element values carried in registers from one pass to a later one
_NO_REUSE_OPS = {"multiply", "mul", "square", "log", "log_fast", "silu", "where"}


def reuse_plan(plan: RowPlan, scalars: dict) -> tuple[dict, dict]:
    """Element values a later pass recomputes exactly as an earlier pass did
    (softmax's exp(x - max) in the sum pass and again in the output pass).

    Every element value gets a structural key: the streamed tensor it loads,
    the per-row values and literals it reads, and the op tree above them.
    Subtrees with products are left out, since whether the assembler
    contracts a product into an add depends on how each name is used.  A
    later Assign whose key matches an earlier pass's value reads that value
    from registers instead of recomputing it; the arithmetic and its order
    are the same, so the bits are.

    Returns ({(pass index, name): slot} for the values to keep,
             {(pass index, name): slot} for the Assigns that reuse them)."""
    row_defs: dict[str, int] = {}
    for st in plan.steps:
        if not isinstance(st, Pass):
            body = st[1] if isinstance(st[1], tuple) else (st[1],)
            for t in ir.walk(body):
                for n in _defines(t):
                    row_defs[n] = row_defs.get(n, 0) + 1
        else:
            for a, _ in st.accs:
                row_defs[a] = row_defs.get(a, 0) + 1
    avail: dict = {}
    keep: dict = {}
    reuse: dict = {}
    passes = [st for st in plan.steps if isinstance(st, Pass)]
    for pi, ps in enumerate(passes):
        keys: dict[str, tuple] = {}
        stmts = list(ir.body_stmts(ps.loop.body))
        counts: dict[str, int] = {}
        for t in stmts:
            for n in _defines(t):
                counts[n] = counts.get(n, 0) + 1

        def key_of(x):
            if not isinstance(x, str):
                return ("num", float(x))
            if x in keys:
                return keys[x]
            if x in row_defs:
                return ("row", x) if row_defs[x] == 1 else None
            if x in scalars:
                return ("scalar", x)
            return None

        for t in stmts:
            if isinstance(t, ir.Load) and t.input in plan.streamed and len(t.names) == 1 \
                    and counts.get(t.names[0]) == 1:
                keys[t.names[0]] = ("load", t.input)
            elif isinstance(t, ir.Let) and isinstance(t.value, ir.Literal) and counts.get(t.name) == 1:
                keys[t.name] = ("lit", float(t.value.value))
            elif isinstance(t, ir.Assign) and counts.get(t.name) == 1:
                op = ir.op_name(t.op)
                ks = [key_of(x) for x in t.args]
                if op in _NO_REUSE_OPS or any(k_ is None for k_ in ks):
                    continue
                k = ("op", op, ir.canon_dtype(t.dtype) if t.dtype is not None else "f32", tuple(ks))
                keys[t.name] = k
                if k in avail and avail[k][0] < pi:
                    src = avail[k]
                    if src not in keep:
                        if len(keep) >= KEEP_MAX:
                            continue
                        keep[src] = len(keep)
                    reuse[(pi, t.name)] = keep[src]
                elif k not in avail and k[1] not in ("copy", "neg", "negative", "abs", "absolute"):
                    avail[k] = (pi, t.name)
    # a reused value that only feeds other reused values is dead in its pass: drop it
    for pi, ps in enumerate(passes):
        stmts = list(ir.body_stmts(ps.loop.body))
        live_reads: set[str] = set()
        for t in stmts:
            if isinstance(t, ir.Assign) and (pi, t.name) in reuse:
                continue
            live_reads |= set(t.reads())
        for t in stmts:
            if isinstance(t, ir.Assign) and (pi, t.name) in reuse and t.name not in live_reads:
                del reuse[(pi, t.name)]
    used = sorted(set(reuse.values()))
    renum = {old: new for new, old in enumerate(used)}
    keep = {src: renum[sl] for src, sl in keep.items() if sl in renum}
    reuse = {k: renum[sl] for k, sl in reuse.items()}
    return keep, reuse


def _stage_bytes(plan: RowPlan, dtypes) -> int:
    return sum(plan.K * ir.ELEM_BYTES[ir.canon_dtype(dtypes.get(n))] for n in plan.streamed)


def _row_loop(plan: RowPlan, shapes, dtypes, ptrs, scalar_env, fus, VW: int, T: int, ind: str,
              bulk: bool = False, reuse_values: bool = True, wr: bool = False) -> list[str]:
    """The persistent loop over this CTA's rows, every pass inside it, for
    vector width VW (4: float4 per access, 1: scalar).  With ``bulk`` the next
    row of every streamed tensor is brought into shared memory by one bulk
    async copy (completion on an mbarrier) while the CTA works on the current
    row from registers."""
    K = plan.K
    nunits = -(-K // VW)
    EPT = -(-nunits // T)
    cached = EPT * VW * max(1, len(plan.streamed)) <= CACHE_FLOATS
    bulk = bulk and cached and VW == 4
    out: list[str] = []
    o = out.append
    if bulk:
        o(f"{ind}uint32_t rn_phase = 0u;")
        o(f"{ind}if (tid == 0 && RB + (long long)blockIdx.x < RE) {{")
        o(f"{ind}    emmy::mbar_arrive_expect_tx(rn_bar, {_stage_bytes(plan, dtypes)}u);")
        for n in plan.streamed:
            dt = ir.canon_dtype(dtypes.get(n))
            o(f"{ind}    emmy::bulk_load(stage_{_c(n)}, {ptrs[n]} + (RB + (long long)blockIdx.x) * K, "
              f"{K * ir.ELEM_BYTES[dt]}u, rn_bar);")
        o(f"{ind}}}")
    if wr:
        o(f"{ind}for (long long row = RB + (long long)blockIdx.x * {WR_ROWS} + wrow; row < RE; "
          f"row += (long long)gridDim.x * {WR_ROWS}) {{")
    else:
        o(f"{ind}for (long long row = RB + blockIdx.x; row < RE; row += gridDim.x) {{")
    i2 = ind + "    "
    # row axes decoded from the flat row index
    rem = "row"
    strides = []
    acc = 1
    for _, e in reversed(plan.row_axes):
        strides.append(acc)
        acc *= e
    strides.reverse()
    row_env = dict(scalar_env)
    # reduction results that divide the row's cells (each is final once folded)
    divisors = {t.args[1] for t in ir.walk(plan.tile.body) if isinstance(t, ir.Assign)
                and ir.op_name(t.op) in DIVIDE_OPS and len(t.args) == 2 and isinstance(t.args[1], str)}
    row_div: dict[str, tuple[str, str]] = {}
    for (name, e), st in zip(plan.row_axes, strides):
        var = f"ra_{_c(name)}"
        expr = f"({rem} / {st}LL) % {e}LL" if st > 1 else f"{rem} % {e}LL"
        o(f"{i2}const long long {var} = {expr};")
        row_env[name] = ("int", var)
    for n in plan.streamed:
        dt = ir.canon_dtype(dtypes.get(n))
        o(f"{i2}const {ctype(dt)} *rp_{_c(n)} = {ptrs[n]} + row * K;")
    for n in plan.outputs:
        dt = ir.canon_dtype(dtypes.get(n))
        o(f"{i2}{ctype(dt)} *rq_{_c(n)} = {ptrs[n]} + row * K;")
    if bulk:
        # this row has landed in shared memory (bounded wait; every thread leaves together)
        o(f"{i2}const bool rn_ok = emmy::mbar_wait(rn_bar, rn_phase, rn_abort, EMMY_STATUS_TIMEOUT_PRODUCER, "
          f"2000000000ull);")
        o(f"{i2}if (__syncthreads_or(!rn_ok)) break;")
        o(f"{i2}rn_phase ^= 1u;")
    if cached:
        for n in plan.streamed:
            dt = ir.canon_dtype(dtypes.get(n))
            if VW == 4:
                o(f"{i2}EmmyVec<{ctype(dt)}, 4> cx_{_c(n)}[{EPT}];")
            else:
                o(f"{i2}{ctype(dt)} cx_{_c(n)}[{EPT}];")
            o(f"{i2}#pragma unroll")
            o(f"{i2}for (int e = 0; e < {EPT}; ++e) {{")
            o(f"{i2}    const long long u = tid + (long long)e * {T};")
            if bulk:
                o(f"{i2}    if (u < {nunits}) cx_{_c(n)}[e] = emmy_lds4_{dt}(stage_{_c(n)} + u * 4);")
            elif VW == 4:
                o(f"{i2}    if (u < {nunits}) cx_{_c(n)}[e] = emmy_ld4_{dt}(rp_{_c(n)} + u * 4, true);")
            else:
                o(f"{i2}    if (u < {nunits}) cx_{_c(n)}[e] = rp_{_c(n)}[u];")
            o(f"{i2}}}")
    if bulk:
        # every thread holds its part of the row: refill the stage with the next row
        o(f"{i2}__syncthreads();")
        o(f"{i2}if (tid == 0 && row + gridDim.x < RE) {{")
        o(f"{i2}    emmy::mbar_arrive_expect_tx(rn_bar, {_stage_bytes(plan, dtypes)}u);")
        for n in plan.streamed:
            dt = ir.canon_dtype(dtypes.get(n))
            o(f"{i2}    emmy::bulk_load(stage_{_c(n)}, {ptrs[n]} + (row + gridDim.x) * K, "
              f"{K * ir.ELEM_BYTES[dt]}u, rn_bar);")
        o(f"{i2}}}")
    declared_row: dict[str, str] = {}
    slot = 0
    keep, reuse = reuse_plan(plan, scalar_env) if cached and reuse_values else ({}, {})
    for k_slot in sorted(set(keep.values())):
        if VW == 4:
            o(f"{i2}EmmyVec<float, 4> kp{k_slot}[{EPT}];")
        else:
            o(f"{i2}float kp{k_slot}[{EPT}];")
    pass_index = -1
    for step in plan.steps:
        if isinstance(step, Pass):
            pass_index += 1
            body = []
            for t in ir.body_stmts(step.loop.body):
                if isinstance(t, ir.Assign) and (pass_index, t.name) in reuse:
                    body.append(ir.Load(names=(t.name,), input=f"__kp{reuse[(pass_index, t.name)]}", index=(),
                                        dtype=ir.DataType("f32", "float32", 4)))
                    continue
                body.append(t)
                if isinstance(t, ir.Assign) and (pass_index, t.name) in keep:
                    body.append(ir.Write(output=f"__kp{keep[(pass_index, t.name)]}", index=(), values=(t.name,),
                                         value_dtype=ir.DataType("f32", "float32", 4)))
            pass_body = tuple(body)
            # per-thread accumulators
            acc_vars = {}
            for a, op in step.accs:
                var = f"acc_{_c(a)}"
                acc_vars[a] = var
                o(f"{i2}float {var} = {f32_lit(identity_of(op))};")
            loop_ind = i2 + "    "
            if cached:
                o(f"{i2}#pragma unroll")
            else:
                o(f"{i2}#pragma unroll 2")
            o(f"{i2}for (int e = 0; e < {EPT}; ++e) {{")
            o(f"{loop_ind}const long long u = tid + (long long)e * {T};")
            o(f"{loop_ind}if (u < {nunits}) {{")
            body_ind = loop_ind + "    "
            # loads that are not per element of a streamed tensor: vectors of [K]
            vec_loaded = {}
            for t in ir.walk(step.loop.body):
                if isinstance(t, ir.Load) and t.input in plan.vectors and t.input not in vec_loaded:
                    dt = ir.canon_dtype(dtypes.get(t.input))
                    vname = f"vv_{_c(t.input)}"
                    if VW == 4:
                        o(f"{body_ind}const auto {vname} = emmy_ld4_{dt}({ptrs[t.input]} + u * 4, false);")
                    else:
                        o(f"{body_ind}const {ctype(dt)} {vname} = {ptrs[t.input]}[u];")
                    vec_loaded[t.input] = vname
                if isinstance(t, ir.Load) and t.input in plan.streamed and not cached and t.input not in vec_loaded:
                    dt = ir.canon_dtype(dtypes.get(t.input))
                    vname = f"sx_{_c(t.input)}"
                    if VW == 4:
                        o(f"{body_ind}const auto {vname} = emmy_ld4_{dt}(rp_{_c(t.input)} + u * 4, false);")
                    else:
                        o(f"{body_ind}const {ctype(dt)} {vname} = rp_{_c(t.input)}[u];")
                    vec_loaded[t.input] = vname
            writes = [t for t in ir.walk(step.loop.body) if isinstance(t, ir.Write)]
            for wi, t in enumerate(writes):
                dt = ir.canon_dtype(dtypes.get(t.output))
                for ln in range(VW):
                    o(f"{body_ind}{ctype(dt)} st{wi}_{ln} = {store_from('f32', '0.0f', dt)};")
            for ln in range(VW):
                def load_hook(s, k, ln=ln):
                    if s.input.startswith("__kp"):  # a value an earlier pass computed
                        return "f32", (f"kp{s.input[4:]}[e].v[{ln}]" if VW == 4 else f"kp{s.input[4:]}[e]")
                    dt = ir.canon_dtype(s.dtype or dtypes.get(s.input))
                    if s.input in plan.streamed:
                        src = f"cx_{_c(s.input)}[e]" if cached else f"sx_{_c(s.input)}"
                    elif s.input in plan.vectors:
                        src = vec_loaded[s.input]
                    else:
                        return em._default_load(s, k)
                    return load_to_kind(f"{src}.v[{ln}]" if VW == 4 else src, dt)

                def write_hook(s, k, kind, code, ln=ln):
                    if s.output.startswith("__kp"):  # kept for a later pass
                        return (f"kp{s.output[4:]}[e].v[{ln}] = {code};" if VW == 4
                                else f"kp{s.output[4:]}[e] = {code};")
                    dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
                    return f"st{writes.index(s)}_{ln} = {store_from(kind, code, dt)};"

                em = Emitter(shapes, dtypes, ptrs, load_hook=load_hook, write_hook=write_hook,
                             indent=body_ind + "    ")
                em.fusable = fus
                em.row_divisors = dict(row_div)
                em.env.update(row_env)
                for a, var in acc_vars.items():
                    em.env[a] = ("f32", var)
                    em.declared[f"{a}|f32"] = var
                for key, var in declared_row.items():
                    em.declared[key] = var
                em.bind_const(step.loop.axis.name, "int", f"(u * {VW}LL + {ln})" if VW == 4 else "u")
                em.run(pass_body)
                o(f"{body_ind}{{")
                out.extend(em.lines)
                o(f"{body_ind}}}")
            for wi, t in enumerate(writes):
                dt = ir.canon_dtype(dtypes.get(t.output))
                if VW == 4:
                    vals = ", ".join(f"st{wi}_{ln}" for ln in range(4))
                    o(f"{body_ind}emmy_st4_{dt}(rq_{_c(t.output)} + u * 4, {vals});")
                else:
                    o(f"{body_ind}rq_{_c(t.output)}[u] = st{wi}_0;")
            o(f"{loop_ind}}}")
            o(f"{i2}}}")
            # block-wide combine: butterfly, one shared stage, every thread folds the
            # warp partials in warp order (same result in every thread, any launch)
            for a, op in step.accs:
                var = acc_vars[a]
                o(f"{i2}#pragma unroll")
                o(f"{i2}for (int off = 16; off > 0; off >>= 1)")
                o(f"{i2}    {var} = {combine_code(op, var, f'__shfl_xor_sync(0xffffffffu, {var}, off)')};")
                if not wr:
                    o(f"{i2}if (lane == 0) red_smem[{slot}][warp] = {var};")
                slot_a = slot
                slot += 1
                acc_vars[a] = (var, slot_a, op)
            if step.accs and not wr:
                o(f"{i2}__syncthreads();")
            for a, (var, sl, op) in acc_vars.items():
                if not wr:
                    # one warp per row: the butterfly left the row's value in every lane
                    o(f"{i2}{var} = red_smem[{sl}][0];")
                    o(f"{i2}#pragma unroll")
                    o(f"{i2}for (int w2 = 1; w2 < {T // 32}; ++w2) {var} = {combine_code(op, var, f'red_smem[{sl}][w2]')};")
                row_env[a] = ("f32", var)
                declared_row[f"{a}|f32"] = var
                if a in divisors:
                    # every cell of the row divides by this value: its reciprocal once per row
                    o(f"{i2}const float rcp_{var} = __frcp_rn({var});")
                    o(f"{i2}const bool dok_{var} = emmy_div_ok({var});")
                    row_div[var] = (f"rcp_{var}", f"dok_{var}")
            continue
        kind, stmt = step
        em = Emitter(shapes, dtypes, ptrs, indent=i2 + ("    " if kind == "leader" else ""))
        em.fusable = fus
        em.row_divisors = dict(row_div)
        em.env.update(row_env)
        for key, var in declared_row.items():
            em.declared[key] = var
        body = stmt if isinstance(stmt, tuple) else (stmt,)
        em.run(body)
        if kind == "leader":
            o(f"{i2}if (tid == 0) {{")
            out.extend(em.lines)
            o(f"{i2}}}")
        else:
            out.extend(em.lines)
            row_env.update({k: v for k, v in em.env.items()})
            declared_row.update(em.declared)
    if wr:
        o(f"{i2}__syncwarp();")
    else:
        o(f"{i2}__syncthreads();  // shared partials are reused by the next row")
    o(f"{ind}}}")
    return out
