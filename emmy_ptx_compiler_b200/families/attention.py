"""Attention family: ``out[i, j] = sum_k w(i, k) * v[k, j]`` where ``w`` comes
from per-key passes over the scores ``s(i, k) = sum_d q[i, d] * kt[d, k]``.

Recognises the naive attention IR (tools/make_proxy_set.py:416-474; lowered
by the reference with compile.py:1813-1864 for every ``Loop``): a Tile over
``(i, j)`` with one thread per output cell, whose body is a sequence of key
loops.  Each key loop recomputes the dot product ``s(i, k)`` with an inner
``Loop`` over ``d`` and then runs a few per-key statements, accumulating
either a per-row value (the row max, the softmax denominator) or the output
cell (the weighted sum of ``v[k, j]``).  Per-row statements (``Init``,
``Let``, ``Assign``, e.g. the reciprocal of the denominator) sit between the
loops, and a final ``Write out[i, j]``.

The reference recomputes every score ``3 x |j|`` times (once per pass and per
output column).  Here a CTA owns ``BQ`` query rows and walks the keys in
tiles of ``BK``:

* all threads compute the tile's ``BQ x BK`` dot products once, sequentially
  over ``d`` with ``fma.rn`` as the reference does, from shared-memory tiles
  of ``q`` and ``kt``; the per-key statements that do not depend on ``j``
  run right there, once per (row, key);
* row accumulations (max, sum) then run in key order by one thread per row,
  so every sum is added in the reference's order;
* the statements that depend on ``j`` (the ``v[k, j]`` product) run in key
  order in the threads that own the output cells, reading ``v`` from a
  shared-memory tile.

Every value is computed with the reference's op table in the reference's
order, FMA contraction included, so results match the reference's PTX to
rounding of its approximate instructions.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .. import ir
from ..cgen import DEVICE_PRELUDE, Emitter, combine_code, ctype, f32_lit, fusable_products
from ..errors import UnsupportedIR
from .common import KernelSource, LaunchPlan, ParamSpec, SM_COUNT, launch_record_source
from .common import c_ident as _c

THREADS = 256
BK = 64
SCORE_CACHE_BYTES = 96 * 1024  # scores of a CTA's rows kept in shared memory across passes
ROWS_PER_CTA = 0               # 0: chosen from the number of query rows
DOT_UNROLL = 16                # unroll of the q . k loop (groups of 4 d)
PV_UNROLL = 16                 # unroll of the p . v loop (groups of 4 keys)
_COMBINE = {"add": "add", "sum": "add", "maximum": "maximum", "amax": "maximum", "max": "maximum",
            "minimum": "minimum", "amin": "minimum", "min": "minimum"}


@dataclass
class KeyLoop:
    loop: ir.Loop
    dot_acc: str            # accumulator of the inner dot product
    dot_init: float
    post: list              # statements after the dot loop
    indep: list             # post statements that do not depend on j
    dep: list               # post statements that depend on j (run by the output owners)
    row_accs: list          # (name, combine op): Accums of j-independent values into per-row state
    stash: list             # j-independent names read by dep statements


@dataclass
class AttnPlan:
    i: str
    j: str
    SQ: int
    DV: int
    SK: int
    D: int
    q: str
    kmat: str
    k_dk: bool              # keys stored [D, SK] (kt) rather than [SK, D]
    v: str | None
    steps: list             # KeyLoop | ("row", stmt)
    out: ir.Write
    out_name: str
    cell_accs: list         # names accumulated per output cell
    notes: dict = field(default_factory=dict)


def _names(index) -> list[str] | None:
    out = []
    for ix in index:
        if not isinstance(ix, ir.Var):
            return None
        out.append(ix.name)
    return out


def _defs(t) -> list[str]:
    if isinstance(t, ir.Load):
        return list(t.names)
    if isinstance(t, (ir.Assign, ir.Let, ir.Init, ir.Accum, ir.Select)):
        return [t.name]
    return []


def match(kop: ir.KernelOp, shapes: dict, dtypes: dict) -> AttnPlan | None:
    body = ir.body_stmts(kop.body)
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        return None
    tile = body[0]
    if len(tile.axes) != 2:
        return None
    (i, SQ), (j, DV) = [(a.name, a.size) for a in tile.axes]
    stmts = list(ir.body_stmts(tile.body))
    loops = [s for s in stmts if isinstance(s, ir.Loop)]
    if len(loops) < 2 or not all(any(isinstance(t, ir.Loop) for t in lp.body) for lp in loops):
        return None
    q = kmat = v = None
    k_dk = None
    SK = D = None
    steps: list = []
    jdep: set[str] = {j}
    cell_accs: list[str] = []
    for s in stmts:
        if isinstance(s, ir.Loop):
            kname = s.axis.name
            ext = s.axis.size
            if SK is None:
                SK = ext
            elif SK != ext:
                return None
            lb = list(s.body)
            inner = [t for t in lb if isinstance(t, ir.Loop)]
            if len(inner) != 1:
                return None
            dl = inner[0]
            pos = lb.index(dl)
            pre = lb[:pos]
            if len(pre) != 1 or not isinstance(pre[0], ir.Init):
                return None
            dot_acc = pre[0].name
            dname = dl.axis.name
            if D is None:
                D = dl.axis.size
            elif D != dl.axis.size:
                return None
            dbody = list(dl.body)
            loads = [t for t in dbody if isinstance(t, ir.Load)]
            accs = [t for t in dbody if isinstance(t, ir.Accum)]
            mults = [t for t in dbody if isinstance(t, ir.Assign)]
            if len(loads) != 2 or len(accs) != 1 or len(dbody) != 4 or len(mults) != 1:
                return None
            mul, acc = mults[0], accs[0]
            if ir.op_name(mul.op) not in ("multiply", "mul") or ir.op_name(acc.op) not in ("add", "sum"):
                return None
            if acc.name != dot_acc or acc.value != mul.name or acc.base not in (None, acc.name):
                return None
            if dbody.index(mul) + 1 != dbody.index(acc):
                return None                      # the reference fuses this pair into fma.rn
            lq = lk = None
            for ld in loads:
                nm = _names(ld.index)
                if nm == [i, dname]:
                    lq = ld
                elif nm in ([dname, kname], [kname, dname]):
                    lk = ld
            if lq is None or lk is None or sorted(mul.args) != sorted([lq.names[0], lk.names[0]]):
                return None
            kd = _names(lk.index) == [dname, kname]
            if q is None:
                q, kmat, k_dk = lq.input, lk.input, kd
            elif (q, kmat, k_dk) != (lq.input, lk.input, kd):
                return None
            post = lb[pos + 1:]
            indep, dep, row_accs = [], [], []
            local_dep: set[str] = set()
            for t in post:
                if not isinstance(t, (ir.Let, ir.Assign, ir.Accum, ir.Load)):
                    return None
                reads = set(t.reads())
                if isinstance(t, ir.Load):
                    nm = _names(t.index)
                    if nm == [kname, j]:
                        if v is None:
                            v = t.input
                        elif v != t.input:
                            return None
                        local_dep |= set(t.names)
                        dep.append(t)
                        continue
                    if nm not in ([kname], [i], [i, kname]) and t.index:
                        return None
                if isinstance(t, ir.Accum):
                    if t.base not in (None, t.name):
                        return None
                    if (reads - {t.name}) & (local_dep | jdep) or t.name in cell_accs:
                        if ir.op_name(t.op) not in ("add", "sum"):
                            return None
                        if t.name not in cell_accs:
                            cell_accs.append(t.name)
                        dep.append(t)
                        jdep.add(t.name)
                        continue
                    op = _COMBINE.get(ir.op_name(t.op))
                    if op is None:
                        return None
                    row_accs.append((t.name, op))
                    continue
                if reads & (local_dep | jdep):
                    local_dep |= set(_defs(t))
                    dep.append(t)
                else:
                    indep.append(t)
            if any(isinstance(t, ir.Accum) for t in indep):
                return None
            own = {a for a, _ in row_accs}
            if any(set(t.reads()) & own for t in indep + [t for t in dep if not isinstance(t, ir.Accum)]):
                return None                      # reads a row value while it is still accumulating
            dep_reads = set()
            for t in dep:
                dep_reads |= set(t.reads())
            stash = [n for n in dict.fromkeys(n for t in indep for n in _defs(t)) if n in dep_reads]
            if dot_acc in dep_reads:
                stash.append(dot_acc)
            steps.append(KeyLoop(s, dot_acc, float(pre[0].identity), post, indep, dep, row_accs, stash))
            continue
        if isinstance(s, ir.Write):
            continue
        if not isinstance(s, (ir.Init, ir.Let, ir.Assign)):
            return None
        if set(s.reads()) & jdep:
            return None
        steps.append(("row", s))
    writes = [s for s in stmts if isinstance(s, ir.Write)]
    if len(writes) != 1 or stmts[-1] is not writes[0]:
        return None
    w = writes[0]
    if _names(w.index) != [i, j] or len(w.values) != 1 or w.atomic:
        return None
    if tuple(shapes.get(w.output, ())) != (SQ, DV):
        return None
    if tuple(shapes.get(q, ())) != (SQ, D):
        return None
    if tuple(shapes.get(kmat, ())) != ((D, SK) if k_dk else (SK, D)):
        return None
    if v is not None and tuple(shapes.get(v, ())) != (SK, DV):
        return None
    for nm in (q, kmat, v, w.output):
        if nm is not None and ir.canon_dtype(dtypes.get(nm)) != "f32":
            raise UnsupportedIR(f"attention on {dtypes.get(nm)} tensor {nm!r} (f32 only)")
    if D > 256 or DV > 256:
        raise UnsupportedIR(f"attention head sizes {D}/{DV} above 256")
    return AttnPlan(i, j, SQ, DV, SK, D, q, kmat, k_dk, v, steps, w, w.output, cell_accs)


def generate(kop: ir.KernelOp, plan: AttnPlan, shapes: dict, dtypes: dict, args: list[str],
             scalars: dict[str, str], written: set[str], first_pass: str = "auto",
             kernel: str = "auto", exchange: str = "auto", tune: dict | None = None) -> KernelSource:
    """``kernel``: "auto" (the tensor-core kernel, families/attention_tc.py,
    when the IR has its shape; else the exact CUDA-core kernel below), "tc"
    or "exact".  ``first_pass`` (exact kernel): "auto" (register-tiled when
    it applies) or "tiled".  ``exchange`` (tensor-core kernel): how the CTAs
    that share a query tile combine their row values, see
    ``attention_tc.layout``; ``tune``: ``attention_tc.TC_TUNE``."""
    if kernel in ("auto", "tc"):
        from . import attention_tc
        lay, why_tc = attention_tc.layout(plan, shapes, dtypes, exchange=exchange)
        if lay is not None:
            return attention_tc.generate_tc(kop, plan, lay, shapes, dtypes, args, scalars, written, tune=tune)
        if kernel == "tc":
            raise UnsupportedIR("no tensor-core attention for this IR: " + "; ".join(why_tc))
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
    SQ, DV, SK, D = plan.SQ, plan.DV, plan.SK, plan.D
    BQ = ROWS_PER_CTA or (16 if -(-SQ // 16) >= 2 * SM_COUNT else (8 if -(-SQ // 8) >= SM_COUNT else 4))
    T = THREADS
    NW = T // 32
    fus = fusable_products(kop.body)
    # per-row names: top-level statements and row accumulators (kept in shared memory per row)
    row_names: list[str] = []
    for st in plan.steps:
        if isinstance(st, KeyLoop):
            for a, _ in st.row_accs:
                if a not in row_names:
                    row_names.append(a)
        else:
            for n in _defs(st[1]):
                if n not in row_names and n not in plan.cell_accs:
                    row_names.append(n)
    nstash = max([len(st.stash) for st in plan.steps if isinstance(st, KeyLoop)] + [0])
    nfac = max([len(st.row_accs) for st in plan.steps if isinstance(st, KeyLoop)] + [0])
    keyloops = [st for st in plan.steps if isinstance(st, KeyLoop)]
    # every key loop computes the same dot products: keep the first pass's scores for the rest
    cache = len(keyloops) > 1 and len({st.dot_init for st in keyloops}) == 1 and BQ * (SK + 4) * 4 <= SCORE_CACHE_BYTES
    # first pass as a register tile: every thread computes all BQ rows for four
    # consecutive keys, reading k straight from L2 (when its values are all that
    # pass keeps: scores for the cache and max / min partials)
    first = keyloops[0] if keyloops else None
    fast1 = (first_pass == "auto" and cache and first is not None and plan.k_dk and D % 4 == 0 and SK % (4 * T) == 0
             and BQ % 4 == 0 and BQ <= 16 and not first.dep and not first.stash
             and all(op in ("maximum", "minimum") for _, op in first.row_accs))
    # the tiles each pass streams through shared memory; passes run one after another,
    # so one double-buffered region holds whatever the pass needs
    need_k = {id(st): not (cache and st is not keyloops[0]) and not (fast1 and st is first) for st in keyloops}
    need_v = {id(st): bool(st.dep and plan.v) for st in keyloops}
    stage = max([(D * BK if need_k[id(st)] else 0) + (BK * DV if need_v[id(st)] else 0) for st in keyloops] + [4])
    stage = -(-stage // 4) * 4
    # 16-byte asynchronous copies when every tile row is whole 16-byte chunks
    # (the kernel also checks the base pointers at run time)
    async_k = plan.k_dk and SK % 4 == 0
    async_v = plan.v is not None and DV % 4 == 0
    q4 = D % 4 == 0
    QS = D if q4 else D + 1     # warps read one q row at a time (broadcast): no padding needed
    SS = BK + 4                 # per-(row, key) operands: float4 rows, rows 4 banks apart
    off = {}
    cur = 0

    def alloc(name, n):
        nonlocal cur
        off[name] = cur
        cur += -(-n // 4) * 4

    SCS = SK + 4                # score-cache row stride: float4-aligned rows, rows 4 banks apart
    alloc("qs", BQ * QS)
    alloc("kv", 2 * stage)
    alloc("rowv", max(1, len(row_names)) * BQ)
    alloc("acca", max(1, nfac) * BQ * SS)   # accumulate operand (or first factor) per (row, key)
    alloc("accb", max(1, nfac) * BQ * SS)   # second factor when the accumulate is an fma
    alloc("stash", max(1, nstash) * BQ * SS)
    np_map = BQ * BK // T if (T % BK == 0 and (BQ * BK) % T == 0) else 1
    alloc("pred", max(1, nfac) * NW * max(1, np_map, BQ if fast1 else 1))   # per-warp partials of max / min rows
    if cache:
        alloc("scache", BQ * SCS)
    smem_bytes = cur * 4
    # CTAs per SM that shared memory allows (1 KiB of it is reserved per CTA), for the register cap
    min_blocks = max(1, min(4, 2048 // T, (228 * 1024) // (smem_bytes + 1024)))
    lines: list[str] = []
    w = lines.append
    w(DEVICE_PRELUDE)
    w('#include "emmy_launch_record.h"')
    w('extern "C" __device__ unsigned int emmy_status;')
    w("__device__ __forceinline__ void emmy_cp16(float *dst, const float *src, unsigned bytes) {")
    w("    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);")
    w('    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(d), "l"(src), "r"(bytes) : "memory");')
    w("}")
    w('__device__ __forceinline__ void emmy_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }')
    w("template <int N> __device__ __forceinline__ void emmy_cp_wait() {")
    w('    asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory");')
    w("}")
    w(f'extern "C" __global__ void __launch_bounds__({T}, {min_blocks}) {kop.name}(' + ", ".join(sig) + ") {")
    w(f"    constexpr int SQ = {SQ}, DV = {DV}, SK = {SK}, D = {D}, BQ = {BQ}, BK = {BK};")
    w(f"    constexpr int QS = {QS}, SS = {SS}, STAGE = {stage}, SCS = {SCS};")
    w(f"    constexpr int NT = (SK + BK - 1) / BK;")
    w("    extern __shared__ __align__(16) float sm[];")
    for name, o in off.items():
        w(f"    float *const {name} = sm + {o};")
    w(f"    uint32_t dyn_smem;")
    w('    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));')
    w(f"    if (blockDim.x != {T} || blockDim.y != 1 || blockDim.z != 1 || dyn_smem < {smem_bytes}u) {{")
    w("        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);")
    w("        return;")
    w("    }")
    w("    const int tid = threadIdx.x;")
    w("    const int lane = tid & 31, warp = tid >> 5;")
    w("    (void)lane; (void)warp;")
    kp, vp = ptrs[plan.kmat], (ptrs[plan.v] if plan.v else None)
    w(f"    const bool k_async = {'true' if async_k else 'false'} && ((reinterpret_cast<uintptr_t>({kp}) & 15) == 0);")
    if plan.v:
        w(f"    const bool v_async = {'true' if async_v else 'false'} && ((reinterpret_cast<uintptr_t>({vp}) & 15) == 0);")
    w("    const long long RB = (long long)(emmy_rb < (unsigned long long)SQ ? emmy_rb : SQ);")
    w("    const long long RE = (long long)(emmy_re < (unsigned long long)SQ ? emmy_re : SQ);")
    w("    for (long long q0 = RB + (long long)blockIdx.x * BQ; q0 < RE; q0 += (long long)gridDim.x * BQ) {")
    w("        const int nq = (RE - q0) < BQ ? (int)(RE - q0) : BQ;")
    w("        __syncthreads();")
    w(f"        for (int e = tid; e < BQ * D; e += {T}) {{")
    w("            const int r = e / D, d = e - r * D;")
    # the fast first pass reads q transposed ([d][row]: one row-quad per float4); no
    # other pass reads q then (the scores are cached)
    qdst = "qs[d * BQ + r]" if fast1 else "qs[r * QS + d]"
    w(f"            {qdst} = r < nq ? {ptrs[plan.q]}[(q0 + r) * D + d] : 0.0f;")
    w("        }")
    # output cell accumulators: thread owns cells o = tid + u*T of the BQ x DV block
    nown = -(-(BQ * DV) // T)
    for a in plan.cell_accs:
        w(f"        float cacc_{_c(a)}[{nown}];")
    row_slot = {n: k for k, n in enumerate(row_names)}

    def row_ref(n: str, r: str) -> str:
        return f"rowv[{row_slot[n]} * BQ + {r}]"

    def tile_load(ind: str, st: KeyLoop, t: str) -> None:
        """Issue the copies of key tile ``t`` into stage ``t & 1`` (asynchronous
        where allowed; plain loads and stores otherwise)."""
        w(f"{ind}{{")
        i1 = ind + "    "
        w(f"{i1}const int tk0 = ({t}) * BK;")
        w(f"{i1}const int tnk = (SK - tk0) < BK ? (SK - tk0) : BK;")
        w(f"{i1}float *const kst = kv + (({t}) & 1) * STAGE;")
        w(f"{i1}(void)tnk; (void)kst;")
        if need_k[id(st)]:
            if plan.k_dk:
                if async_k:
                    w(f"{i1}if (k_async) {{")
                    w(f"{i1}    for (int e = tid; e < D * (BK / 4); e += {T}) {{")
                    w(f"{i1}        const int d = e / (BK / 4), kk = (e - d * (BK / 4)) * 4;")
                    w(f"{i1}        const bool in = kk < tnk;")
                    w(f"{i1}        emmy_cp16(kst + d * BK + kk, {kp} + (in ? (long long)d * SK + tk0 + kk : 0), in ? 16u : 0u);")
                    w(f"{i1}    }}")
                    w(f"{i1}}} else")
                w(f"{i1}for (int e = tid; e < D * BK; e += {T}) {{")
                w(f"{i1}    const int d = e / BK, kk = e - d * BK;")
                w(f"{i1}    kst[d * BK + kk] = kk < tnk ? {kp}[(long long)d * SK + tk0 + kk] : 0.0f;")
                w(f"{i1}}}")
            else:
                w(f"{i1}for (int e = tid; e < D * BK; e += {T}) {{")
                w(f"{i1}    const int kk = e / D, d = e - kk * D;")
                w(f"{i1}    kst[d * BK + kk] = kk < tnk ? {kp}[(long long)(tk0 + kk) * D + d] : 0.0f;")
                w(f"{i1}}}")
        if need_v[id(st)]:
            voff = D * BK if need_k[id(st)] else 0
            w(f"{i1}float *const vst = kst + {voff};")
            if async_v:
                w(f"{i1}if (v_async) {{")
                w(f"{i1}    for (int e = tid; e < BK * (DV / 4); e += {T}) {{")
                w(f"{i1}        const int kk = e / (DV / 4), jj = (e - kk * (DV / 4)) * 4;")
                w(f"{i1}        const bool in = kk < tnk;")
                w(f"{i1}        emmy_cp16(vst + kk * DV + jj, {vp} + (in ? (long long)(tk0 + kk) * DV + jj : 0), in ? 16u : 0u);")
                w(f"{i1}    }}")
                w(f"{i1}}} else")
            w(f"{i1}for (int e = tid; e < BK * DV; e += {T}) {{")
            w(f"{i1}    const int kk = e / DV, jj = e - kk * DV;")
            w(f"{i1}    vst[kk * DV + jj] = kk < tnk ? {vp}[(long long)(tk0 + kk) * DV + jj] : 0.0f;")
            w(f"{i1}}}")
        w(f"{ind}}}")

    ind = "        "
    for st in plan.steps:
        if not isinstance(st, KeyLoop):
            s = st[1]
            # per-row statement: thread r < BQ computes it for row r
            if isinstance(s, ir.Init) and s.name in plan.cell_accs:
                for u in range(nown):
                    w(f"{ind}cacc_{_c(s.name)}[{u}] = {f32_lit(float(s.identity))};")
                continue
            w(f"{ind}__syncthreads();")
            w(f"{ind}if (tid < BQ) {{")
            em = Emitter(shapes, dtypes, ptrs, indent=ind + "    ")
            em.fusable = fus
            em.env.update(scalar_env)
            em.bind_const(plan.i, "int", "(q0 + tid)")
            for n in row_names:
                if n in row_slot and _row_defined(plan, n, st):
                    em.env[n] = ("f32", row_ref(n, "tid"))
            em.run((s,))
            w("\n".join(em.lines))
            for n in _defs(s):
                if n in row_slot:
                    w(f"{ind}    {row_ref(n, 'tid')} = {em.as_f32(n)};")
            w(f"{ind}}}")
            continue
        if fast1 and st is first:
            _emit_fast_first_pass(w, ind, st, plan, shapes, dtypes, ptrs, fus, scalar_env, row_names, row_ref,
                                  BQ, T, NW, SK, D)
            continue
        reuse = cache and st is not keyloops[0]
        loads = need_k[id(st)] or need_v[id(st)]
        # (row, key) pairs: thread tid takes key kk = tid % BK of rows tid / BK + u * RS,
        # the same rows on every tile (so it can keep per-row partials in registers)
        mapped = T % BK == 0 and (BQ * BK) % T == 0 and BK % 32 == 0
        NP = BQ * BK // T if mapped else 0
        RS = T // BK if mapped else 0
        acc_kinds = []                 # (fi, name, op, kind): kind "reg", "fma" or "smem"
        for fi, (a, op) in enumerate(st.row_accs):
            accum = next(t for t in st.post if isinstance(t, ir.Accum) and t.name == a)
            if mapped and op in ("maximum", "minimum"):
                acc_kinds.append((fi, a, op, "reg", accum))
            else:
                acc_kinds.append((fi, a, op, "fma" if op == "add" else "smem", accum))
        reg_accs = [k for k in acc_kinds if k[3] == "reg"]
        smem_accs = [k for k in acc_kinds if k[3] != "reg"]
        phase2 = bool(smem_accs or st.dep)
        # the previous pass's readers of the stage buffers and row values are done
        w(f"{ind}__syncthreads();")
        for ri, (fi, a, op, _, _) in enumerate(reg_accs):
            # per-thread partial of a max / min: same value in any order of keys
            w(f"{ind}float pm{ri}[{NP}];")
            w(f"{ind}#pragma unroll")
            w(f"{ind}for (int u = 0; u < {NP}; ++u) pm{ri}[u] = {row_ref(a, f'(tid / BK + u * {RS})')};")
        if loads:
            tile_load(ind, st, "0")
            w(f"{ind}emmy_cp_commit();")
        w(f"{ind}for (int t = 0; t < NT; ++t) {{")
        i2 = ind + "    "
        w(f"{i2}const int k0 = t * BK;")
        w(f"{i2}const int nk = (SK - k0) < BK ? (SK - k0) : BK;")
        if loads:
            w(f"{i2}emmy_cp_wait<0>();")
        if loads or phase2:
            # tile t is visible to all; every thread is done with tile t - 1
            w(f"{i2}__syncthreads();")
        if loads:
            # the next tile streams into the other stage while this one is used
            w(f"{i2}if (t + 1 < NT) {{")
            tile_load(i2 + "    ", st, "t + 1")
            w(f"{i2}    emmy_cp_commit();")
            w(f"{i2}}}")
        w(f"{i2}const float *const ks = kv + (t & 1) * STAGE;")
        w(f"{i2}const float *const vs = ks + {D * BK if need_k[id(st)] else 0};")
        w(f"{i2}(void)ks; (void)vs;")
        # scores and j-independent statements, once per (row, key)
        i3 = i2 + "    "
        if mapped:
            w(f"{i2}{{")
            w(f"{i3}const int kk = tid % BK;")
            if not reuse:
                # each k element read from shared memory feeds NP rows' fma chains
                # (each still sequential over d)
                w(f"{i3}float scv[{NP}];")
                w(f"{i3}#pragma unroll")
                w(f"{i3}for (int u = 0; u < {NP}; ++u) scv[u] = {f32_lit(st.dot_init)};")
                w(f"{i3}if (kk < nk) {{")
                if q4:
                    w(f"{i3}    #pragma unroll {DOT_UNROLL}")
                    w(f"{i3}    for (int d4 = 0; d4 < D; d4 += 4) {{")
                    w(f"{i3}        float4 qv[{NP}];")
                    w(f"{i3}        #pragma unroll")
                    w(f"{i3}        for (int u = 0; u < {NP}; ++u)")
                    w(f"{i3}            qv[u] = *reinterpret_cast<const float4 *>(qs + (tid / BK + u * {RS}) * QS + d4);")
                    w(f"{i3}        const float k0v = ks[(d4 + 0) * BK + kk], k1v = ks[(d4 + 1) * BK + kk];")
                    w(f"{i3}        const float k2v = ks[(d4 + 2) * BK + kk], k3v = ks[(d4 + 3) * BK + kk];")
                    w(f"{i3}        #pragma unroll")
                    w(f"{i3}        for (int u = 0; u < {NP}; ++u) {{")
                    w(f"{i3}            scv[u] = __fmaf_rn(qv[u].x, k0v, scv[u]);")
                    w(f"{i3}            scv[u] = __fmaf_rn(qv[u].y, k1v, scv[u]);")
                    w(f"{i3}            scv[u] = __fmaf_rn(qv[u].z, k2v, scv[u]);")
                    w(f"{i3}            scv[u] = __fmaf_rn(qv[u].w, k3v, scv[u]);")
                    w(f"{i3}        }}")
                    w(f"{i3}    }}")
                else:
                    w(f"{i3}    #pragma unroll 4")
                    w(f"{i3}    for (int d = 0; d < D; ++d) {{")
                    w(f"{i3}        const float kv_ = ks[d * BK + kk];")
                    w(f"{i3}        #pragma unroll")
                    w(f"{i3}        for (int u = 0; u < {NP}; ++u)")
                    w(f"{i3}            scv[u] = __fmaf_rn(qs[(tid / BK + u * {RS}) * QS + d], kv_, scv[u]);")
                    w(f"{i3}    }}")
                w(f"{i3}}}")
            w(f"{i3}#pragma unroll")
            w(f"{i3}for (int u = 0; u < {NP}; ++u) {{")
            w(f"{i3}const int r = tid / BK + u * {RS};")
        else:
            w(f"{i2}for (int p = tid; p < BQ * BK; p += {T}) {{")
            w(f"{i3}const int r = p / BK, kk = p - r * BK;")
        w(f"{i3}if (r < nq && kk < nk) {{")
        i4 = i3 + "    "
        if reuse:
            w(f"{i4}float sc = scache[r * SCS + k0 + kk];")
        elif mapped:
            w(f"{i4}float sc = scv[u];")
            if cache:
                w(f"{i4}scache[r * SCS + k0 + kk] = sc;")
        else:
            w(f"{i4}float sc = {f32_lit(st.dot_init)};")
            w(f"{i4}#pragma unroll 8")
            w(f"{i4}for (int d = 0; d < D; ++d) sc = __fmaf_rn(qs[r * QS + d], ks[d * BK + kk], sc);")
            if cache:
                w(f"{i4}scache[r * SCS + k0 + kk] = sc;")
        em = Emitter(shapes, dtypes, ptrs, indent=i4)
        em.fusable = fus
        em.env.update(scalar_env)
        em.bind_const(plan.i, "int", "(q0 + r)")
        em.bind_const(st.loop.axis.name, "int", "(k0 + kk)")
        em.env[st.dot_acc] = ("f32", "sc")
        em.declared[f"{st.dot_acc}|f32"] = "sc"
        for n in row_names:
            em.env.setdefault(n, ("f32", row_ref(n, "r")))
        em.run(tuple(st.indep))
        w("\n".join(em.lines))
        # fold the register partials; stash the accumulate operands and the values
        # the j-dependent statements read
        acc_ops = []
        for ri, (fi, a, op, kind, accum) in enumerate(reg_accs):
            w(f"{i4}pm{ri}[u] = {combine_code(op, f'pm{ri}[u]', em.as_f32(accum.value))};")
        for fi, a, op, kind, accum in smem_accs:
            prod = em.plain_product(accum.value) if op == "add" else None
            if prod is not None:
                w(f"{i4}acca[({fi} * BQ + r) * SS + kk] = {prod[0]};")
                w(f"{i4}accb[({fi} * BQ + r) * SS + kk] = {prod[1]};")
                acc_ops.append((fi, a, op, True))
            else:
                w(f"{i4}acca[({fi} * BQ + r) * SS + kk] = {em.as_f32(accum.value)};")
                acc_ops.append((fi, a, op, False))
        stash_codes = {}
        for si, n in enumerate(st.stash):
            w(f"{i4}stash[({si} * BQ + r) * SS + kk] = {em.as_f32(n)};")
            stash_codes[n] = si
        w(f"{i3}}}")
        w(f"{i2}}}")
        if mapped:
            w(f"{i2}}}")
        if phase2:
            w(f"{i2}__syncthreads();")
        # row accumulations kept in shared memory.  max / min give the same value in
        # any order: one warp per row combines the tile in parallel.  Sums run in key
        # order, one thread per row, so every sum is added in the reference's order.
        # The statements that depend on j read no accumulator of this loop, so they
        # run alongside.
        for fi, a, op, is_fma in acc_ops:
            acc_at = f"acca[({fi} * BQ + r) * SS + kk]"
            if op in ("maximum", "minimum") and not is_fma:
                w(f"{i2}for (int r = warp; r < nq; r += {NW}) {{")
                w(f"{i2}    float x = {row_ref(a, 'r')};")
                w(f"{i2}    for (int kk = lane; kk < nk; kk += 32) x = {combine_code(op, 'x', acc_at)};")
                w(f"{i2}    #pragma unroll")
                w(f"{i2}    for (int o = 16; o > 0; o >>= 1) x = {combine_code(op, 'x', '__shfl_xor_sync(0xffffffffu, x, o)')};")
                w(f"{i2}    __syncwarp();")
                w(f"{i2}    if (lane == 0) {row_ref(a, 'r')} = x;")
                w(f"{i2}}}")
                continue
            w(f"{i2}if (tid < nq) {{")
            w(f"{i2}    const int r = tid;")
            w(f"{i2}    float ra = {row_ref(a, 'r')};")
            if is_fma:
                step = f"ra = __fmaf_rn({acc_at}, accb[({fi} * BQ + r) * SS + kk], ra);"
            else:
                step = f"ra = {combine_code(op, 'ra', acc_at)};"
            w(f"{i2}    if (nk == BK) {{")
            w(f"{i2}        #pragma unroll 16")
            w(f"{i2}        for (int kk = 0; kk < BK; ++kk) {step}")
            w(f"{i2}    }} else {{")
            w(f"{i2}        for (int kk = 0; kk < nk; ++kk) {step}")
            w(f"{i2}    }}")
            w(f"{i2}    {row_ref(a, 'r')} = ra;")
            w(f"{i2}}}")
        # j-dependent statements in key order, in the threads that own the output cells
        if st.dep:
            _emit_dep(w, i2, st, plan, shapes, dtypes, ptrs, fus, scalar_env, row_names, row_ref,
                      stash_codes, nown, T)
        w(f"{ind}}}")
        if reg_accs:
            # combine the partials of each row: over the lanes of a warp, then over the
            # BK / 32 warps that hold the row
            for ri, (fi, a, op, kind, accum) in enumerate(reg_accs):
                w(f"{ind}#pragma unroll")
                w(f"{ind}for (int u = 0; u < {NP}; ++u) {{")
                w(f"{ind}    float x = pm{ri}[u];")
                w(f"{ind}    #pragma unroll")
                w(f"{ind}    for (int o = 16; o > 0; o >>= 1) x = {combine_code(op, 'x', '__shfl_xor_sync(0xffffffffu, x, o)')};")
                w(f"{ind}    if (lane == 0) pred[({ri} * {NW} + warp) * {NP} + u] = x;")
                w(f"{ind}}}")
            w(f"{ind}__syncthreads();")
            w(f"{ind}if (tid < nq) {{")
            w(f"{ind}    const int r = tid, u = r / {RS}, w0 = (r % {RS}) * (BK / 32);")
            for ri, (fi, a, op, kind, accum) in enumerate(reg_accs):
                w(f"{ind}    {{")
                w(f"{ind}        float x = {row_ref(a, 'r')};")
                w(f"{ind}        for (int wv = w0; wv < w0 + BK / 32; ++wv) x = {combine_code(op, 'x', f'pred[({ri} * {NW} + wv) * {NP} + u]')};")
                w(f"{ind}        {row_ref(a, 'r')} = x;")
                w(f"{ind}    }}")
            w(f"{ind}}}")
    # the output (row values may come from a row statement of another thread)
    w(f"{ind}__syncthreads();")
    w(f"{ind}#pragma unroll")
    w(f"{ind}for (int u = 0; u < {nown}; ++u) {{")
    w(f"{ind}    const int o = tid + u * {T};")
    w(f"{ind}    const int r = o / DV, jj = o - r * DV;")
    w(f"{ind}    if (r < nq) {{")
    val = plan.out.values[0]
    if val in plan.cell_accs:
        code = f"cacc_{_c(val)}[u]"
    elif val in row_slot:
        code = row_ref(val, "r")
    else:
        raise UnsupportedIR(f"attention output {val!r} is neither a cell nor a row value")
    w(f"{ind}        {ptrs[plan.out_name]}[(q0 + r) * DV + jj] = {code};")
    w(f"{ind}    }}")
    w(f"{ind}}}")
    w("    }")
    w("}")
    blocks = -(-SQ // BQ)
    grid = max(1, min(blocks, SM_COUNT * 8))
    rb = []
    for name in args:
        if name in (plan.q,):
            rb.append(D * 4)
        elif name == plan.out_name:
            rb.append(DV * 4)
        else:
            rb.append(0)
    launch = LaunchPlan(grid=(grid, 1, 1), block=(T, 1, 1), smem=smem_bytes, range_total=SQ, range_align=BQ,
                        range_bytes=rb)
    lines.append(launch_record_source("attention", launch, params))
    notes = {"kernel": "attention_rows", "rows_per_cta": BQ, "key_tile": BK, "threads": T, "score_cache": cache,
             "register_tiled_first_pass": fast1,
             "passes": len(keyloops), "smem": smem_bytes, "async_k": async_k, "async_v": async_v,
             "min_blocks": min_blocks}
    return KernelSource(entry=kop.name, source="\n".join(lines), launch=launch, params=params,
                        family="attention", notes=notes)


def _emit_fast_first_pass(w, ind, st, plan, shapes, dtypes, ptrs, fus, scalar_env, row_names, row_ref,
                          BQ, T, NW, SK, D) -> None:
    """The first key loop as a register tile: thread t owns keys kb * 4T + 4t .. +3
    of every key block kb and all BQ rows, 4 * BQ independent fma chains, each
    still sequential over d as the reference computes it.  k is read from L2 one
    float4 (four keys) per d; q comes transposed from shared memory, one
    broadcast float4 per four rows.  Scores go to the cache; the row max / min
    stays in registers and is combined across threads once."""
    kp = ptrs[plan.kmat]
    w(f"{ind}__syncthreads();")
    for ri, (a, op) in enumerate(st.row_accs):
        w(f"{ind}float fm{ri}[BQ];")
        w(f"{ind}#pragma unroll")
        w(f"{ind}for (int r = 0; r < BQ; ++r) fm{ri}[r] = {row_ref(a, 'r')};")
    w(f"{ind}const bool k_vec = ((reinterpret_cast<uintptr_t>({kp}) & 15) == 0);")
    w(f"{ind}for (int kb = 0; kb < SK / (4 * {T}); ++kb) {{")
    i2 = ind + "    "
    w(f"{i2}const int kbase = kb * (4 * {T}) + 4 * tid;")
    w(f"{i2}const float *const kcol = {kp} + kbase;")
    w(f"{i2}float sv[BQ][4];")
    w(f"{i2}#pragma unroll")
    w(f"{i2}for (int r = 0; r < BQ; ++r) {{ sv[r][0] = sv[r][1] = sv[r][2] = sv[r][3] = {f32_lit(st.dot_init)}; }}")
    w(f"{i2}#pragma unroll 8")
    w(f"{i2}for (int d = 0; d < D; ++d) {{")
    w(f"{i2}    const float *const kd = kcol + (long long)d * SK;")
    w(f"{i2}    const float4 kv4 = k_vec ? *reinterpret_cast<const float4 *>(kd) : make_float4(kd[0], kd[1], kd[2], kd[3]);")
    w(f"{i2}    #pragma unroll")
    w(f"{i2}    for (int r4 = 0; r4 < BQ; r4 += 4) {{")
    w(f"{i2}        const float4 q4 = *reinterpret_cast<const float4 *>(qs + d * BQ + r4);")
    for rr, qc in enumerate(("x", "y", "z", "w")):
        for c, kc in enumerate(("x", "y", "z", "w")):
            w(f"{i2}        sv[r4 + {rr}][{c}] = __fmaf_rn(q4.{qc}, kv4.{kc}, sv[r4 + {rr}][{c}]);")
    w(f"{i2}    }}")
    w(f"{i2}}}")
    w(f"{i2}#pragma unroll")
    w(f"{i2}for (int r = 0; r < BQ; ++r) {{")
    w(f"{i2}    #pragma unroll")
    w(f"{i2}    for (int c = 0; c < 4; ++c) {{")
    w(f"{i2}        if (r < nq) {{")
    i5 = i2 + "            "
    w(f"{i5}const int kk = kbase + c;")
    w(f"{i5}float sc = sv[r][c];")
    w(f"{i5}scache[r * SCS + kk] = sc;")
    em = Emitter(shapes, dtypes, ptrs, indent=i5)
    em.fusable = fus
    em.env.update(scalar_env)
    em.bind_const(plan.i, "int", "(q0 + r)")
    em.bind_const(st.loop.axis.name, "int", "(long long)kk")
    em.env[st.dot_acc] = ("f32", "sc")
    em.declared[f"{st.dot_acc}|f32"] = "sc"
    for n in row_names:
        em.env.setdefault(n, ("f32", row_ref(n, "r")))
    em.run(tuple(st.indep))
    w("\n".join(em.lines))
    for ri, (a, op) in enumerate(st.row_accs):
        accum = next(t for t in st.post if isinstance(t, ir.Accum) and t.name == a)
        w(f"{i5}fm{ri}[r] = {combine_code(op, f'fm{ri}[r]', em.as_f32(accum.value))};")
    w(f"{i2}        }}")
    w(f"{i2}    }}")
    w(f"{i2}}}")
    w(f"{ind}}}")
    # every thread holds a partial of every row: over the warp, then over the warps
    for ri, (a, op) in enumerate(st.row_accs):
        w(f"{ind}#pragma unroll")
        w(f"{ind}for (int r = 0; r < BQ; ++r) {{")
        w(f"{ind}    float x = fm{ri}[r];")
        w(f"{ind}    #pragma unroll")
        w(f"{ind}    for (int o = 16; o > 0; o >>= 1) x = {combine_code(op, 'x', '__shfl_xor_sync(0xffffffffu, x, o)')};")
        w(f"{ind}    if (lane == 0) pred[({ri} * {NW} + warp) * BQ + r] = x;")
        w(f"{ind}}}")
    if st.row_accs:
        w(f"{ind}__syncthreads();")
        w(f"{ind}if (tid < nq) {{")
        for ri, (a, op) in enumerate(st.row_accs):
            w(f"{ind}    {{")
            w(f"{ind}        float x = {row_ref(a, 'tid')};")
            w(f"{ind}        for (int wv = 0; wv < {NW}; ++wv) x = {combine_code(op, 'x', f'pred[({ri} * {NW} + wv) * BQ + tid]')};")
            w(f"{ind}        {row_ref(a, 'tid')} = x;")
            w(f"{ind}    }}")
        w(f"{ind}}}")


def _emit_dep(w, i2, st, plan, shapes, dtypes, ptrs, fus, scalar_env, row_names, row_ref, stash_codes,
              nown, T) -> None:
    """The statements of a key loop that depend on ``j`` (the ``v[k, j]``
    product and the cell accumulation), in key order per output cell."""
    DV = plan.DV

    def run(indent, load_code, stash_code):
        em2 = Emitter(shapes, dtypes, ptrs, indent=indent, load_hook=lambda s_, k_: ("f32", load_code))
        em2.fusable = fus
        em2.env.update(scalar_env)
        em2.bind_const(plan.i, "int", "(q0 + r)")
        em2.bind_const(plan.j, "int", "jj")
        em2.bind_const(st.loop.axis.name, "int", "(k0 + kk)")
        for n in row_names:
            em2.env.setdefault(n, ("f32", row_ref(n, "r")))
        for n, si in stash_codes.items():
            em2.env[n] = ("f32", stash_code(si))
        for a in plan.cell_accs:
            em2.env[a] = ("f32", f"cacc_{_c(a)}[u]")
            em2.declared[f"{a}|f32"] = f"cacc_{_c(a)}[u]"
        em2.run(tuple(st.dep))
        w("\n".join(em2.lines))

    ns = len(stash_codes)
    if T % DV == 0:
        # every owned cell of a thread has the same column: one v read per key feeds
        # them all; full tiles read each row's stashed values four keys at a time
        w(f"{i2}{{")
        w(f"{i2}const int jj = tid % DV;")
        if ns:
            w(f"{i2}if (nk == BK) {{")
            w(f"{i2}    #pragma unroll {PV_UNROLL}")
            w(f"{i2}    for (int k4 = 0; k4 < BK; k4 += 4) {{")
            w(f"{i2}        float wst[{ns}][{nown}][4];")
            w(f"{i2}        #pragma unroll")
            w(f"{i2}        for (int u = 0; u < {nown}; ++u) {{")
            w(f"{i2}            const int r = (tid + u * {T}) / DV;")
            for si in range(ns):
                w(f"{i2}            const float4 t{si} = r < nq ? *reinterpret_cast<const float4 *>(stash + ({si} * BQ + r) * SS + k4) : make_float4(0.f, 0.f, 0.f, 0.f);")
                w(f"{i2}            wst[{si}][u][0] = t{si}.x; wst[{si}][u][1] = t{si}.y; wst[{si}][u][2] = t{si}.z; wst[{si}][u][3] = t{si}.w;")
            w(f"{i2}        }}")
            w(f"{i2}        #pragma unroll")
            w(f"{i2}        for (int c = 0; c < 4; ++c) {{")
            w(f"{i2}            const int kk = k4 + c;")
            w(f"{i2}            const float vcur = vs[kk * DV + jj];")
            w(f"{i2}            #pragma unroll")
            w(f"{i2}            for (int u = 0; u < {nown}; ++u) {{")
            w(f"{i2}                const int r = (tid + u * {T}) / DV;")
            w(f"{i2}                if (r < nq) {{")
            run(i2 + "                    ", "vcur", lambda si: f"wst[{si}][u][c]")
            w(f"{i2}                }}")
            w(f"{i2}            }}")
            w(f"{i2}        }}")
            w(f"{i2}    }}")
            w(f"{i2}}} else")
        w(f"{i2}for (int kk = 0; kk < nk; ++kk) {{")
        w(f"{i2}    const float vcur = vs[kk * DV + jj];")
        w(f"{i2}    #pragma unroll")
        w(f"{i2}    for (int u = 0; u < {nown}; ++u) {{")
        w(f"{i2}        const int r = (tid + u * {T}) / DV;")
        w(f"{i2}        if (r < nq) {{")
        run(i2 + "            ", "vcur", lambda si: f"stash[({si} * BQ + r) * SS + kk]")
        w(f"{i2}        }}")
        w(f"{i2}    }}")
        w(f"{i2}}}")
        w(f"{i2}}}")
        return
    w(f"{i2}#pragma unroll")
    w(f"{i2}for (int u = 0; u < {nown}; ++u) {{")
    w(f"{i2}    const int o = tid + u * {T};")
    w(f"{i2}    const int r = o / DV, jj = o - r * DV;")
    w(f"{i2}    if (r < nq) {{")
    w(f"{i2}        for (int kk = 0; kk < nk; ++kk) {{")
    run(i2 + "            ", "vs[kk * DV + jj]", lambda si: f"stash[({si} * BQ + r) * SS + kk]")
    w(f"{i2}        }}")
    w(f"{i2}    }}")
    w(f"{i2}}}")


def _row_defined(plan: AttnPlan, name: str, upto) -> bool:
    """Whether ``name`` already holds a value in shared memory before step ``upto``."""
    for st in plan.steps:
        if st is upto:
            return False
        if isinstance(st, KeyLoop):
            if name in [a for a, _ in st.row_accs]:
                return True
        elif name in _defs(st[1]):
            return True
    return False
