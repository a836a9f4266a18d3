"""Reduction family: ``out[row] = post(combine_k f(x[row, k]))``.

Recognises the reduction schedules the reference lowers
(tools/make_proxy_set.py:215-336, tools/make_world_set.py:247-266):

* the cooperative strided schedule: a Tile over ``(rows..., co)`` whose body
  is ``StridedLoop(k, start=co, step=|co|)`` accumulating, then
  ``WarpShuffle`` + per-warp ``Smem`` + ``Sync`` + ``TreeHalve``
  (compile.py:1866-1914, 2213-2286), optional post-ops and the ``co == 0``
  write;
* one thread per row with a plain ``Loop`` over k (compile.py:1813-1864);
* a pointwise body whose only output is an atomic ``red.global.add`` into a
  scalar (compile.py:2035-2039), i.e. a full sum.

The reference runs a row on one 128-thread block and a full-array sum on a
single block (grid [1,1,1]).  This family instead splits every row into
``CH`` chunks so that rows x chunks fill all 148 SMs, streams each chunk with
128-bit loads (four 16-byte loads in flight per thread), reduces a chunk with
``__shfl_xor_sync`` butterflies plus one shared-memory stage and one barrier,
and combines a row's chunk partials in a fixed order in whichever block
finishes that row last (a per-row arrival counter).  Results therefore do not
depend on the grid size or on block scheduling, only on the block size.

Accumulator seeds and combine ops follow the reference (identity_of,
compile.py:327-338; Accum, compile.py:2201-2211), including the
``multiply`` -> ``Accum add`` FMA contraction (compile.py:1263-1283).
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

from .. import ir
from ..cgen import (DEVICE_PRELUDE, Emitter, combine_code, ctype, f32_lit, identity_of, load_to_kind,
                    lit_int)
from ..errors import UnsupportedIR
from .common import KernelSource, LaunchPlan, ParamSpec, SM_COUNT, launch_record_source
from .common import c_ident as _c

BLOCK = 256
UNROLL = 4
VEC = 4
BLOCKS_PER_SM = 8
MIN_CHUNK = BLOCK * VEC * UNROLL * 4
_SCHEDULE = (ir.WarpShuffle, ir.TreeHalve, ir.Smem, ir.Sync)
_ELEM = (ir.Load, ir.Let, ir.Init, ir.Assign, ir.Accum, ir.Select, ir.Cond)


@dataclass
class ReductionPlan:
    kind: str                      # "strided" | "loop" | "atomic"
    row_axes: list[tuple[str, int]]
    red_axes: list[tuple[str, int]]
    elem_body: tuple
    accs: list[tuple[str, str]]    # (name, combine op) in order of appearance
    seeds: dict[str, float]
    pre_body: tuple
    post_body: tuple
    atomic_write: ir.Write | None = None
    notes: dict = field(default_factory=dict)

    @property
    def rows(self) -> int:
        n = 1
        for _, e in self.row_axes:
            n *= e
        return n

    @property
    def klen(self) -> int:
        n = 1
        for _, e in self.red_axes:
            n *= e
        return n


def _accums(body) -> list[tuple[str, str]]:
    out: list[tuple[str, str]] = []
    for s in ir.walk(body):
        if isinstance(s, ir.Accum) and s.name not in [a for a, _ in out]:
            if s.base not in (None, s.name):
                raise UnsupportedIR("Accum with a foreign base is not a reduction")
            out.append((s.name, ir.op_name(s.op)))
    return out


def _only(body, types) -> bool:
    return all(isinstance(s, types) for s in ir.walk(body))


def _unwrap_leader(stmt, co: str):
    """``Cond(co == 0, body)`` -> body (the one-writer epilogue of the schedule)."""
    if isinstance(stmt, ir.Cond) and not stmt.else_body and isinstance(stmt.cond, ir.BinaryExpr):
        c = stmt.cond
        if c.op == "==" and isinstance(c.left, ir.Var) and c.left.name == co and lit_int(c.right) == 0:
            return stmt.body
    return None


def _smem_write_cond(stmt, smem_names: set[str]) -> bool:
    if not isinstance(stmt, ir.Cond):
        return False
    inner = list(ir.walk(stmt.body)) + list(ir.walk(stmt.else_body))
    return bool(inner) and all(isinstance(t, ir.Write) and t.output in smem_names for t in inner)


def _check_combines(stmts, accs: dict[str, str]) -> None:
    for s in stmts:
        if isinstance(s, (ir.WarpShuffle, ir.TreeHalve)):
            for c in s.combine_states:
                if not isinstance(c, ir.Assign):
                    raise UnsupportedIR("reduction combine is not an Assign")
                op = ir.op_name(c.op)
                if c.name not in accs:
                    raise UnsupportedIR(f"combine of unknown state {c.name!r}")
                if op != accs[c.name] and not ({op, accs[c.name]} <= {"add", "sum"}):
                    raise UnsupportedIR(f"combine op {op} disagrees with accumulate op {accs[c.name]}")


def match(kop: ir.KernelOp, shapes: dict, dtypes: dict) -> ReductionPlan | None:
    body = ir.body_stmts(kop.body)
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        return None
    tile = body[0]
    stmts = list(ir.body_stmts(tile.body))
    axes = [(a.name, a.size) for a in tile.axes]
    strided = [s for s in stmts if isinstance(s, ir.StridedLoop)]
    loops = [s for s in stmts if isinstance(s, ir.Loop)]
    if strided and not loops and len(strided) == 1:
        return _match_strided(tile, stmts, axes, strided[0])
    if loops and not strided and len(loops) == 1:
        return _match_loop(stmts, axes, loops[0])
    atomics = [s for s in ir.walk(tile.body) if isinstance(s, ir.Write) and s.atomic]
    if atomics and not strided and not loops:
        return _match_atomic(stmts, axes, atomics)
    return None


def _match_strided(tile, stmts, axes, loop: ir.StridedLoop) -> ReductionPlan | None:
    if not axes:
        return None
    co, co_ext = axes[-1]
    step = lit_int(loop.step)
    if not (isinstance(loop.start, ir.Var) and loop.start.name == co and step == co_ext):
        return None
    end = loop.axis.size if loop.end is None else lit_int(loop.end)
    if end is None:
        raise UnsupportedIR("StridedLoop end is not a constant")
    if not _only(loop.body, _ELEM):
        raise UnsupportedIR("reduction loop body has non-elementwise statements")
    accs = _accums(loop.body)
    if not accs:
        return None
    i = stmts.index(loop)
    pre = tuple(stmts[:i])
    if not _only(pre, (ir.Init, ir.Let, ir.Smem)):
        raise UnsupportedIR("statements before the reduction loop are not seeds")
    smem_names = {s.name for s in ir.walk(tile.body) if isinstance(s, ir.Smem)}
    sched, post = [], []
    for s in stmts[i + 1:]:
        if isinstance(s, _SCHEDULE) or _smem_write_cond(s, smem_names):
            sched.append(s)
            continue
        lead = _unwrap_leader(s, co)
        post.extend(lead if lead is not None else (s,))
    _check_combines(sched, dict(accs))
    for s in post:
        for t in ir.walk((s,)):
            if isinstance(t, ir.Load) and t.input in smem_names:
                raise UnsupportedIR("post-reduction read of shared memory")
            if isinstance(t, (ir.Loop, ir.StridedLoop, *_SCHEDULE)):
                raise UnsupportedIR("loop after the reduction (fused row-reduce + pointwise)")
            for v in (t.reads() if isinstance(t, ir.Stmt) else ()):
                if v == co:
                    raise UnsupportedIR("post-reduction code reads the cooperative thread axis")
    seeds = _seeds(pre, accs, strict=True)
    red_axes = [(loop.axis.name, end)]
    return ReductionPlan("strided", axes[:-1], red_axes, loop.body, accs, seeds, pre, tuple(post))


def _match_loop(stmts, axes, loop: ir.Loop) -> ReductionPlan | None:
    if not _only(loop.body, _ELEM):
        return None
    accs = _accums(loop.body)
    if not accs:
        return None
    i = stmts.index(loop)
    pre = tuple(stmts[:i])
    post = tuple(stmts[i + 1:])
    if not _only(pre, (ir.Init, ir.Let)):
        return None
    if not _only(post, (ir.Load, ir.Let, ir.Assign, ir.Write, ir.Select, ir.Cond)):
        return None
    seeds = _seeds(pre, accs, strict=False)
    return ReductionPlan("loop", axes, [(loop.axis.name, loop.axis.size)], loop.body, accs, seeds, pre,
                         post)


def _match_atomic(stmts, axes, atomics) -> ReductionPlan | None:
    if len(atomics) != 1 or atomics[0].index or len(atomics[0].values) != 1:
        return None
    w = atomics[0]
    # ZeroPrologue (compile.py:2890-2913): the kernel itself zero-fills `words`
    # 32-bit words of a buffer before accumulating into it
    zps = [s for s in stmts if isinstance(s, ir.ZeroPrologue)]
    elem = tuple(s for s in stmts if s is not w and not isinstance(s, ir.ZeroPrologue))
    if w not in stmts or not _only(elem, (ir.Load, ir.Let, ir.Assign, ir.Select)):
        return None
    acc = "__atomic_total"
    elem = elem + (ir.Accum(acc, w.values[0], ir.ElementwiseImpl("add"), None),)
    plan = ReductionPlan("atomic", [], axes, elem, [(acc, "add")], {}, (), (), atomic_write=w)
    plan.notes["zero_prologue"] = [(z.dst, int(lit_int(z.words) if not isinstance(z.words, int) else z.words))
                                   for z in zps]
    return plan


def _seeds(pre, accs, strict: bool) -> dict[str, float]:
    seeds: dict[str, float] = {}
    names = dict(accs)
    for s in pre:
        if isinstance(s, ir.Init) and s.name in names:
            v = float(s.identity)
            if strict and v != identity_of(names[s.name]):
                raise UnsupportedIR("cooperative reduction seeded with a non-identity value")
            seeds[s.name] = v
    return seeds


# ---------------------------------------------------------------------------- codegen


def _vector_layout(plan: ReductionPlan, shapes, dtypes) -> tuple[bool, list[str]]:
    """Vector path: every element Load is f32 and addresses (rows..., k),
    (rows...) or (k) with unit stride along k; K % 4 == 0."""
    why: list[str] = []
    if plan.kind == "atomic" or len(plan.red_axes) != 1:
        why.append("flattened multi-axis reduction")
        return False, why
    k_name, klen = plan.red_axes[0]
    if klen % VEC:
        why.append(f"reduction extent {klen} is not a multiple of {VEC}")
    rows = [a for a, _ in plan.row_axes]
    for s in ir.walk(plan.elem_body):
        if isinstance(s, ir.Cond):
            why.append("Cond in the element body")
        if isinstance(s, ir.Load):
            dt = ir.canon_dtype(s.dtype or dtypes.get(s.input))
            names = [ix.name if isinstance(ix, ir.Var) else None for ix in s.index]
            if len(s.names) != 1 or dt != "f32":
                why.append(f"Load {s.input} is not a single f32")
            elif names == rows + [k_name] and tuple(shapes.get(s.input, ())) == tuple(
                    [e for _, e in plan.row_axes] + [klen]):
                pass
            elif names == [k_name] and tuple(shapes.get(s.input, ())) in ((klen,), ()):
                pass
            elif names == rows and rows:
                pass
            else:
                why.append(f"Load {s.input} index is not (rows..., k)")
    return (not why), why


def _pick_chunks(rows: int, klen: int) -> tuple[int, int]:
    """Chunks per row: rows of at least two MIN_CHUNKs split in two from half
    a wave of rows up (8192, 4096, 2048 and 1024 rows of 65536 f32: 6.9, 6.7,
    6.2 and 5.9 TB/s against 6.5, 6.5, 5.8 and 5.4 with one CTA per row; four
    chunks measured below two); fewer rows split into as many chunks as fill
    one wave, each at least MIN_CHUNK long."""
    target = SM_COUNT * BLOCKS_PER_SM
    if klen <= MIN_CHUNK:
        return 1, klen
    if rows >= target // 2:
        ch = min(2, klen // MIN_CHUNK)
        if ch == 1:
            return 1, klen
    else:
        ch = min(-(-target // rows), max(1, klen // MIN_CHUNK))
    length = -(-klen // ch)
    length = -(-length // (VEC * 32)) * (VEC * 32)
    ch = -(-klen // length)
    return ch, length


def generate(kop: ir.KernelOp, plan: ReductionPlan, shapes: dict, dtypes: dict, args: list[str],
             scalars: dict[str, str], written: set[str]) -> KernelSource:
    vec_ok, why = _vector_layout(plan, shapes, dtypes)
    rows, klen = plan.rows, plan.klen
    ch, chunk = _pick_chunks(rows, klen)
    nacc = len(plan.accs)
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
    scalar_env = {n: (("f32", f"p_{_c(n)}") if scalars[n] == "f32" else ("int", f"(long long)p_{_c(n)}"))
                  for n in scalars}
    accs = plan.accs
    # a full-array reduction can combine its result across GPUs at the end of
    # the kernel (<name>__xchg, emmy_xchg_dev.cuh); the body then takes the
    # exchange parameter, NULL in the single-GPU entry
    xchg = (rows == 1 and plan.kind != "atomic" and 1 <= nacc <= XCHG_MAX_VALUES
            and all(op in XCHG_OPS for _, op in accs))
    L: list[str] = []
    w = L.append
    w(DEVICE_PRELUDE)
    w(_RED_HELPERS)
    if xchg:
        w('#include "emmy_xchg_dev.cuh"')
        L.extend(_xchg_function(accs, _c(kop.name)))
    if ch > 1:
        w(f"__device__ float emmy_red_partials[{nacc * rows * ch}];")
        w(f"__device__ unsigned int emmy_red_arrivals[{rows}];")
    body_fn = f"emmy_red_body_{_c(kop.name)}"
    if xchg:
        w(f"static __device__ __forceinline__ void {body_fn}(" + ", ".join(sig + ["const EmmyXchgArgs *emmy_xa"])
          + ") {")
    else:
        w(f'extern "C" __global__ void __launch_bounds__(1024) {kop.name}(' + ", ".join(sig) + ") {")
    w(f"    constexpr long long ROWS = {rows}LL, KLEN = {klen}LL, CH = {ch}LL, CHUNK = {chunk}LL;")
    w("    constexpr int NACC = %d;" % nacc)
    w("    if ((blockDim.x & 31u) != 0u || blockDim.y != 1u || blockDim.z != 1u) {")
    w("        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);")
    w("        return;")
    w("    }")
    w("    __shared__ float s_warp[NACC][32];")
    w("    __shared__ int s_last;")
    w("    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nwarps = blockDim.x >> 5;")
    if vec_ok:
        aligned = " | ".join(f"(uintptr_t){p}" for p in ptrs.values()) or "0"
        w(f"    const bool vec_ok = (({aligned}) & 15u) == 0;")
    w("    for (long long vb = blockIdx.x; vb < ROWS * CH; vb += gridDim.x) {")
    w("        const long long row = vb / CH, chunk = vb % CH;")
    w("        const long long k0 = chunk * CHUNK;")
    w("        const long long k1 = (k0 + CHUNK < KLEN) ? (k0 + CHUNK) : KLEN;")
    for a, op in accs:
        ident = f32_lit(identity_of(op))
        for u in range(UNROLL):
            w(f"        float pa_{_c(a)}_{u} = {ident};")
    row_env = _row_decode(plan, "        ")
    L.extend(row_env)
    if vec_ok:
        w("        if (vec_ok) {")
        w(f"            long long k = k0 + (long long)tid * {VEC};")
        w(f"            const long long kstep = (long long)blockDim.x * {VEC};")
        w(f"            for (; k + {UNROLL - 1} * kstep < k1; k += {UNROLL} * kstep) {{")
        L.extend(_vec_trip(plan, shapes, dtypes, ptrs, scalar_env, list(range(UNROLL)), "                "))
        w("            }")
        w("            for (; k < k1; k += kstep) {")
        L.extend(_vec_trip(plan, shapes, dtypes, ptrs, scalar_env, [0], "                "))
        w("            }")
        w("        } else")
    w("        {")
    w("            long long k = k0 + tid;")
    w("            const long long kstep = blockDim.x;")
    w(f"            for (; k + {UNROLL - 1} * kstep < k1; k += {UNROLL} * kstep) {{")
    for u in range(UNROLL):
        L.extend(_scalar_elem(plan, shapes, dtypes, ptrs, scalar_env, u, f"k + {u} * kstep",
                              "                "))
    w("            }")
    w("            for (; k < k1; k += kstep) {")
    L.extend(_scalar_elem(plan, shapes, dtypes, ptrs, scalar_env, 0, "k", "                "))
    w("            }")
    w("        }")
    # in-thread, warp and block combine (fixed order)
    for a, op in accs:
        t = f"t_{_c(a)}"
        w(f"        float {t} = {combine_code(op, f'pa_{_c(a)}_0', f'pa_{_c(a)}_1')};")
        w(f"        {t} = {combine_code(op, t, combine_code(op, f'pa_{_c(a)}_2', f'pa_{_c(a)}_3'))};")
        w(f"        for (int off = 16; off > 0; off >>= 1) {t} = {combine_code(op, t, f'__shfl_xor_sync(0xffffffffu, {t}, off)')};")
    w("        if (lane == 0) {")
    for i, (a, _) in enumerate(accs):
        w(f"            s_warp[{i}][wid] = t_{_c(a)};")
    w("        }")
    w("        __syncthreads();")
    w("        if (wid == 0) {")
    for i, (a, op) in enumerate(accs):
        ident = f32_lit(identity_of(op))
        w(f"            float b_{_c(a)} = lane < nwarps ? s_warp[{i}][lane] : {ident};")
        w(f"            for (int off = 16; off > 0; off >>= 1) b_{_c(a)} = {combine_code(op, f'b_{_c(a)}', f'__shfl_xor_sync(0xffffffffu, b_{_c(a)}, off)')};")
    if ch == 1:
        w("            if (lane == 0) {")
        if xchg:
            L.extend(_xchg_combine(accs, "b_", "                ", _c(kop.name)))
        L.extend(_epilogue(plan, shapes, dtypes, ptrs, scalar_env, {a: f"b_{_c(a)}" for a, _ in accs},
                           "                "))
        w("            }")
        w("        }")
        w("        __syncthreads();")
    else:
        w("            if (lane == 0) {")
        for i, (a, _) in enumerate(accs):
            w(f"                __stcg(&emmy_red_partials[({i} * ROWS + row) * CH + chunk], b_{_c(a)});")
        w("                __threadfence();")
        w("                const unsigned prev = atomicAdd(&emmy_red_arrivals[row], 1u);")
        w("                s_last = (prev == (unsigned)(CH - 1));")
        w("            }")
        w("        }")
        w("        __syncthreads();")
        w("        if (s_last) {")
        w("            __threadfence();")
        for i, (a, op) in enumerate(accs):
            ident = f32_lit(identity_of(op))
            w(f"            float c_{_c(a)} = {ident};")
            w(f"            for (long long c = tid; c < CH; c += blockDim.x) c_{_c(a)} = {combine_code(op, f'c_{_c(a)}', f'__ldcg(&emmy_red_partials[({i} * ROWS + row) * CH + c])')};")
            w(f"            for (int off = 16; off > 0; off >>= 1) c_{_c(a)} = {combine_code(op, f'c_{_c(a)}', f'__shfl_xor_sync(0xffffffffu, c_{_c(a)}, off)')};")
        w("            __syncthreads();")
        w("            if (lane == 0) {")
        for i, (a, _) in enumerate(accs):
            w(f"                s_warp[{i}][wid] = c_{_c(a)};")
        w("            }")
        w("            __syncthreads();")
        w("            if (wid == 0) {")
        for i, (a, op) in enumerate(accs):
            ident = f32_lit(identity_of(op))
            w(f"                float f_{_c(a)} = lane < nwarps ? s_warp[{i}][lane] : {ident};")
            w(f"                for (int off = 16; off > 0; off >>= 1) f_{_c(a)} = {combine_code(op, f'f_{_c(a)}', f'__shfl_xor_sync(0xffffffffu, f_{_c(a)}, off)')};")
        w("                if (lane == 0) {")
        if xchg:
            L.extend(_xchg_combine(accs, "f_", "                    ", _c(kop.name)))
        L.extend(_epilogue(plan, shapes, dtypes, ptrs, scalar_env, {a: f"f_{_c(a)}" for a, _ in accs},
                           "                    "))
        w("                    emmy_red_arrivals[row] = 0u;")
        w("                }")
        w("            }")
        w("        }")
        w("        __syncthreads();")
    w("    }")
    w("}")
    if xchg:
        names = ", ".join(s_.split()[-1] for s_ in sig)
        w(f'extern "C" __global__ void __launch_bounds__(1024) {kop.name}(' + ", ".join(sig) + ") {")
        w(f"    {body_fn}({names}{', ' if names else ''}nullptr);")
        w("}")
        w(f'extern "C" __global__ void __launch_bounds__(1024) {kop.name}__xchg('
          + ", ".join(sig + ["const __grid_constant__ EmmyXchgArgs emmy_xa"]) + ") {")
        w(f"    {body_fn}({names}{', ' if names else ''}&emmy_xa);")
        w("}")
    nvb = rows * ch
    grid = max(1, min(nvb, SM_COUNT * BLOCKS_PER_SM))
    launch = LaunchPlan(grid=(grid, 1, 1), block=(BLOCK, 1, 1), smem=0)
    L.append(launch_record_source("reduction", launch, params))
    notes = {"vector": vec_ok, "scalar_reasons": why, "rows": rows, "klen": klen, "chunks": ch,
             "chunk_len": chunk, "schedule": plan.kind, "accumulators": [a for a, _ in accs],
             "cross_gpu_entry": f"{kop.name}__xchg" if xchg else None}
    return KernelSource(entry=kop.name, source="\n".join(L), launch=launch, params=params,
                        family="reduction", notes=notes)


XCHG_MAX_VALUES = 4
XCHG_OPS = ("add", "sum", "max", "maximum", "amax", "min", "minimum", "amin")


def _xchg_function(accs, name: str) -> list[str]:
    """A separate (not inlined) device function for the cross-GPU combine, so the
    exchange's arrays do not weigh on the register allocation of the streaming
    loop: every GPU's values exchanged, each accumulator's combined in rank
    order (NaN when the exchange failed)."""
    lanes = "xyzw"
    out = [f"static __device__ __noinline__ float4 emmy_red_combine_{name}(const EmmyXchgArgs *xa, float4 in) {{",
           f"    const float v[4] = {{in.x, in.y, in.z, in.w}};",
           f"    float g[{len(accs)} * EMMY_XCHG_MAX_RANKS_DEV];",
           "    float4 out = in;",
           f"    if (!emmy_xchg_exchange(*xa, v, {len(accs)}, g)) {{",
           "        const float nan = __int_as_float(0x7fffffff);",
           "        return make_float4(nan, nan, nan, nan);",
           "    }"]
    for i, (a, op) in enumerate(accs):
        out += ["    {",
                f"        float c = g[{i} * xa->nranks];",
                f"        for (unsigned r = 1; r < xa->nranks; ++r) c = {combine_code(op, 'c', f'g[{i} * xa->nranks + r]')};",
                f"        out.{lanes[i]} = c;",
                "    }"]
    out += ["    return out;", "}"]
    return out


def _xchg_combine(accs, prefix: str, ind: str, name: str) -> list[str]:
    """In the thread holding the row's final values: with an exchange
    parameter, replace each value by the combine of every GPU's value."""
    lanes = "xyzw"
    vals = [prefix + _c(a) for a, _ in accs] + ["0.0f"] * (4 - len(accs))
    out = [f"{ind}if (emmy_xa) {{",
           f"{ind}    const float4 emmy_r = emmy_red_combine_{name}(emmy_xa, make_float4({', '.join(vals)}));"]
    for i, (a, _) in enumerate(accs):
        out.append(f"{ind}    {prefix}{_c(a)} = emmy_r.{lanes[i]};")
    out.append(f"{ind}}}")
    return out


def _row_decode(plan: ReductionPlan, ind: str) -> list[str]:
    out = []
    strides = []
    acc = 1
    for _, e in reversed(plan.row_axes):
        strides.append(acc)
        acc *= e
    strides.reverse()
    for i, ((name, e), st) in enumerate(zip(plan.row_axes, strides)):
        q = "row" if st == 1 else f"(row / {st}LL)"
        expr = q if i == 0 else f"({q} % {e}LL)"
        out.append(f"{ind}const long long r_{i} = {expr};")
    return out


def _bind_rows(em: Emitter, plan: ReductionPlan) -> None:
    for i, (name, _) in enumerate(plan.row_axes):
        em.bind_const(name, "int", f"r_{i}")


def _elem_emitter(plan, shapes, dtypes, ptrs, scalar_env, u: int, ind: str, load_hook=None) -> Emitter:
    em = Emitter(shapes, dtypes, ptrs, load_hook=load_hook, indent=ind)
    em.env.update(scalar_env)
    _bind_rows(em, plan)
    for a, _ in plan.accs:
        var = f"pa_{_c(a)}_{u}"
        em.env[a] = ("f32", var)
        em.declared[f"{a}|f32"] = var
    return em


def _scalar_elem(plan, shapes, dtypes, ptrs, scalar_env, u: int, kexpr: str, ind: str) -> list[str]:
    em = _elem_emitter(plan, shapes, dtypes, ptrs, scalar_env, u, ind + "    ")
    em.emit(f"const long long kk = {kexpr};")
    if plan.kind == "atomic":
        strides = []
        acc = 1
        for _, e in reversed(plan.red_axes):
            strides.append(acc)
            acc *= e
        strides.reverse()
        for i, ((name, e), st) in enumerate(zip(plan.red_axes, strides)):
            q = "kk" if st == 1 else f"(kk / {st}LL)"
            expr = q if i == 0 else f"({q} % {e}LL)"
            em.emit(f"const long long kx_{i} = {expr};")
            em.bind_const(name, "int", f"kx_{i}")
    else:
        em.bind_const(plan.red_axes[0][0], "int", "kk")
    em.run(plan.elem_body)
    return [ind + "{"] + em.lines + [ind + "}"]


def _vec_trip(plan, shapes, dtypes, ptrs, scalar_env, us: list[int], ind: str) -> list[str]:
    out: list[str] = []
    k_name, klen = plan.red_axes[0]
    rows = [a for a, _ in plan.row_axes]
    row_strides = []
    acc = 1
    for _, e in reversed(plan.row_axes):
        row_strides.append(acc)
        acc *= e
    row_strides.reverse()
    row_flat = " + ".join(f"r_{i} * {st}LL" for i, st in enumerate(row_strides)) or "0LL"
    loads = [s for s in ir.walk(plan.elem_body) if isinstance(s, ir.Load)]
    for u in us:
        out.append(f"{ind}const long long kv{u} = k + {u} * kstep;")
        for li, s in enumerate(loads):
            names = [ix.name if isinstance(ix, ir.Var) else None for ix in s.index]
            ptr = ptrs[s.input]
            if names == rows + [k_name]:
                out.append(f"{ind}const float4 g{li}_{u} = __ldcs(reinterpret_cast<const float4*>({ptr} + ({row_flat}) * {klen}LL + kv{u}));")
            elif names == [k_name]:
                out.append(f"{ind}const float4 g{li}_{u} = __ldg(reinterpret_cast<const float4*>({ptr} + kv{u}));")
            else:
                out.append(f"{ind}const float g{li}_{u} = {ptr}[{row_flat}];")
    load_idx = {id(s): li for li, s in enumerate(loads)}
    for u in us:
        for lane, comp in enumerate("xyzw"):
            def hook(s, k, u=u, comp=comp):
                names = [ix.name if isinstance(ix, ir.Var) else None for ix in s.index]
                li = load_idx[id(s)]
                if names == rows and rows and names != rows + [k_name]:
                    return load_to_kind(f"g{li}_{u}", "f32")
                return load_to_kind(f"g{li}_{u}.{comp}", "f32")
            em = _elem_emitter(plan, shapes, dtypes, ptrs, scalar_env, u, ind + "    ", load_hook=hook)
            em.bind_const(k_name, "int", f"(kv{u} + {lane})")
            em.run(plan.elem_body)
            out.append(ind + "{")
            out.extend(em.lines)
            out.append(ind + "}")
    return out


def _epilogue(plan, shapes, dtypes, ptrs, scalar_env, totals: dict[str, str], ind: str) -> list[str]:
    def write_hook(s, k, kind, code):
        dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
        idx = em.flat_index(s.output, em.index_plus(s.index, k))
        if plan.kind == "atomic":
            return f"{ptrs[s.output]}[{idx}] = __fadd_rn({ptrs[s.output]}[{idx}], {em._to_f32(kind, code)});"
        from ..cgen import store_from
        return f"{ptrs[s.output]}[{idx}] = {store_from(kind, code, dt)};"

    em = Emitter(shapes, dtypes, ptrs, write_hook=write_hook, indent=ind)
    em.env.update(scalar_env)
    _bind_rows(em, plan)
    for a, op in plan.accs:
        total = totals[a]
        seed = plan.seeds.get(a)
        if plan.kind == "loop" and seed is not None and seed != identity_of(op):
            total = combine_code(op, f32_lit(seed), total)
        em.assign(a, "f32", total)
    if plan.kind == "atomic":
        w = plan.atomic_write
        # the zero fill comes first: no block writes these buffers before the final combine
        for dst, words in plan.notes.get("zero_prologue", []):
            if dst in ptrs and words > 0:
                em.emit(f"for (int zw = 0; zw < {words}; ++zw) reinterpret_cast<unsigned *>({ptrs[dst]})[zw] = 0u;")
        em.stmt(ir.Write(w.output, (), (plan.accs[0][0],), w.value_dtype, False))
    else:
        em.run(plan.post_body)
    return em.lines


_RED_HELPERS = r"""
#include "emmy_launch_record.h"
extern "C" __device__ unsigned int emmy_status;
"""
