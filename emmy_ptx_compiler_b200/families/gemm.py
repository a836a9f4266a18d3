"""GEMM family: ``C[i, j] = epilogue(sum_k A[i, k] * B[k, j])``.

Recognises the reference's naive matmul schedule (tools/make_proxy_set.py:
338-365): a Tile over (i, j), ``Init acc``, ``Loop(kk)`` with two Loads, a
``multiply`` and an ``Accum add`` (the reference lowers it to one thread per
output running ``fma.rn.f32`` over k, compile.py:1813-1864, 1263-1283),
followed by per-output epilogue statements (bias add, ReLU, ... ) and the
Write of C.

Two kernels:

* ``tcgen05`` - bf16/fp16 operands, fp32 accumulation on the 5th-generation
  tensor cores.  Persistent, warp-specialised CTAs of 192 threads: warp 0
  issues TMA tile loads (128x64 of A, 64x256 of B, 128-byte swizzle) into a
  4-stage mbarrier ring, warp 1 allocates 512 TMEM columns and issues
  ``tcgen05.mma.cta_group::1.kind::f16`` 128x256x16 instructions into one of
  two TMEM accumulators, warps 2-5 drain the other accumulator with
  ``tcgen05.ld``, run the IR's epilogue in registers and store C - so the
  epilogue of tile t overlaps the main loop of tile t+1.  Every wait is
  bounded (a timeout raises a status bit instead of hanging).  Needs K and,
  for a [K, N] B, N to be multiples of 8 (16-byte TMA strides).
* ``simt`` - everything else (f32 operands, ragged strides): shared-memory
  tiles and CUDA-core FMAs, each output accumulated in k order exactly as the
  reference's loop does, so f32 results match the reference PTX bit for bit.
"""

from __future__ import annotations

import re
from dataclasses import dataclass

from .. import ir
from ..cgen import DEVICE_PRELUDE, Emitter, ctype, f32_lit, store_from
from ..errors import UnsupportedIR
from .common import KernelSource, LaunchPlan, ParamSpec, SM_COUNT, TmapSpec, launch_record_source
from .common import c_ident as _c

BM, BN, BK, STAGES = 128, 256, 64, 4
PAIR_BM, PAIR_STAGES = 256, 6   # CTA-pair tile: 256 x 256, 128 rows and 128 B-columns per CTA
TC_THREADS = 192
SIMT_BM, SIMT_BN, SIMT_BK, SIMT_THREADS = 64, 64, 16, 256
GROUP_M = 16
# CTA-pair kernel schedule knobs (results do not depend on them): row-tiles per
# column sweep, C stores ("wb" write-back, "cs" streaming), L2 policies of the
# A and B tile loads (None, "evict_last", "evict_first")
PAIR_TUNE = {"group_m": 8, "c_store": "wb", "a_policy": None, "b_policy": None,
             # failure-detection tests only: a shorter limit for every bounded wait, and a
             # producer that leaves out its first TMA load (CTA 1 of cluster 0, first tile),
             # so that the leader's stage never fills and the bounded waits run out
             "wait_ns": 2000000000, "skip_first_load": False}
TMAP_DTYPE = {"bf16": 9, "f16": 6}
SWIZZLE_128B = 3
L2_256B = 3


@dataclass
class GemmPlan:
    i: str
    j: str
    k: str
    M: int
    N: int
    K: int
    a: ir.Load
    b: ir.Load
    b_nk: bool            # B stored [N, K] (K-major) instead of [K, N]
    acc: str
    seed: float
    epilogue: tuple
    out: ir.Write | None
    ab_dtype: str


def _var_names(index) -> list[str] | None:
    out = []
    for ix in index:
        if not isinstance(ix, ir.Var):
            return None
        out.append(ix.name)
    return out


def match(kop: ir.KernelOp, shapes: dict, dtypes: dict) -> GemmPlan | None:
    body = ir.body_stmts(kop.body)
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        return None
    tile = body[0]
    if len(tile.axes) != 2:
        return None
    (i, M), (j, N) = [(a.name, a.size) for a in tile.axes]
    stmts = list(ir.body_stmts(tile.body))
    loops = [s for s in stmts if isinstance(s, ir.Loop)]
    if len(loops) != 1 or any(isinstance(s, ir.StridedLoop) for s in stmts):
        return None
    loop = loops[0]
    k, K = loop.axis.name, loop.axis.size
    lb = list(ir.body_stmts(loop.body))
    if len(lb) != 4 or not all(isinstance(s, ir.Load) for s in lb[:2]):
        return None
    l0, l1, mul, acc = lb
    if not (isinstance(mul, ir.Assign) and ir.op_name(mul.op) == "multiply" and len(mul.args) == 2
            and isinstance(acc, ir.Accum) and ir.op_name(acc.op) in ("add", "sum") and acc.value == mul.name
            and acc.base in (None, acc.name) and set(mul.args) == {l0.names[0], l1.names[0]}
            and len(l0.names) == 1 and len(l1.names) == 1):
        return None
    n0, n1 = _var_names(l0.index), _var_names(l1.index)
    if n0 is None or n1 is None:
        return None
    if n0 == [i, k]:
        a, b, nb = l0, l1, n1
    elif n1 == [i, k]:
        a, b, nb = l1, l0, n0
    else:
        return None
    if nb == [k, j]:
        b_nk = False
    elif nb == [j, k]:
        b_nk = True
    else:
        return None
    if tuple(shapes.get(a.input, (M, K))) != (M, K):
        return None
    if tuple(shapes.get(b.input, ())) != ((N, K) if b_nk else (K, N)):
        return None
    li = stmts.index(loop)
    seed = 0.0
    for s in stmts[:li]:
        if isinstance(s, ir.Init) and s.name == acc.name:
            seed = float(s.identity)
        elif not isinstance(s, (ir.Init, ir.Let)):
            return None
    epi = tuple(stmts[li + 1:])
    for s in ir.walk(epi):
        if isinstance(s, (ir.Loop, ir.StridedLoop, ir.Accum, ir.Smem, ir.Sync, ir.WarpShuffle, ir.TreeHalve)):
            return None
        if isinstance(s, ir.Write) and s.atomic:
            return None
    writes = [s for s in ir.walk(epi) if isinstance(s, ir.Write)]
    if not writes:
        return None
    out = None
    if (len(writes) == 1 and writes[0] in epi and _var_names(writes[0].index) == [i, j]
            and len(writes[0].values) == 1 and tuple(shapes.get(writes[0].output, (M, N))) == (M, N)):
        out = writes[0]
    adt = ir.canon_dtype(a.dtype or dtypes.get(a.input))
    bdt = ir.canon_dtype(b.dtype or dtypes.get(b.input))
    if adt != bdt or adt not in ("f32", "bf16", "f16"):
        raise UnsupportedIR(f"GEMM operands {adt} x {bdt} (need matching f32, bf16 or f16)")
    return GemmPlan(i, j, k, M, N, K, a, b, b_nk, acc.name, seed, epi, out, adt)


def range_bytes(plan: GemmPlan, args: list[str], shapes: dict, dtypes: dict, scalars: dict) -> list[int] | None:
    """Bytes per output row of each parameter for row-range launches: A's row
    (K elements) and C's row (N elements); everything else is read whole.
    None when the epilogue writes anything but C[i, j] of an [M, N] buffer."""
    if plan.out is None:
        return None
    for s in ir.walk(plan.epilogue):
        if isinstance(s, ir.Write) and s is not plan.out:
            return None
    out = []
    for name in args:
        if name in scalars:
            out.append(0)
        elif name == plan.a.input and tuple(shapes.get(name, ())) == (plan.M, plan.K) and name != plan.out.output:
            out.append(plan.K * ir.ELEM_BYTES.get(ir.canon_dtype(dtypes.get(name)), 4))
        elif name == plan.out.output and tuple(shapes.get(name, ())) == (plan.M, plan.N):
            out.append(plan.N * ir.ELEM_BYTES.get(ir.canon_dtype(dtypes.get(name)), 4))
        else:
            out.append(0)
    return out


RANGE_SIG = ["unsigned long long emmy_rb", "unsigned long long emmy_re"]


def _row_range(tile_rows: int, mb_total: int) -> str:
    """Kernel prologue: this launch's rows [RB, RE) as row-tiles [MB0, MB0 + MBN)."""
    return (f"    const long long RB = (long long)(emmy_rb < (unsigned long long)M ? emmy_rb : M);\n"
            f"    const long long RE = (long long)(emmy_re < (unsigned long long)M ? emmy_re : M);\n"
            f"    const int MB0 = (int)(RB / {tile_rows});\n"
            f"    const int MBN = RE > RB ? (int)((RE + {tile_rows} - 1) / {tile_rows}) - MB0 : 0;\n"
            f"    const int TILES = MBN * NB;\n")


def _tc_ok(plan: GemmPlan, dtypes) -> tuple[bool, list[str]]:
    why = []
    if plan.ab_dtype not in ("bf16", "f16"):
        why.append(f"{plan.ab_dtype} operands run on CUDA cores (tcgen05 kind::f16 needs bf16/f16)")
    if plan.K % 8:
        why.append(f"K={plan.K} is not a multiple of 8 (16-byte TMA row stride)")
    if not plan.b_nk and plan.N % 8:
        why.append(f"N={plan.N} is not a multiple of 8 (16-byte TMA row stride of B)")
    if plan.out is None:
        why.append("epilogue does not write exactly one C[i, j]")
    else:
        odt = ir.canon_dtype(plan.out.value_dtype or dtypes.get(plan.out.output))
        if odt not in ("bf16", "f16", "f32"):
            why.append(f"output type {odt}")
    if plan.seed != 0.0:
        why.append("non-zero accumulator seed")
    return (not why), why


def generate(kop: ir.KernelOp, plan: GemmPlan, shapes: dict, dtypes: dict, args: list[str],
             scalars: dict[str, str], written: set[str], *, variant: str = "auto",
             tune: dict | None = None, meta_threads: int = 0) -> KernelSource:
    """``variant``: "auto" (CTA-pair kernel when M >= 256 and N >= 256, else
    single-CTA), "pair", "single"; non-TMA-able shapes and f32 go to SIMT."""
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
    # every GEMM module takes a row range after its tensor maps (rows it cannot
    # stream are then marked 0 bytes per row: read or written whole)
    rbytes = range_bytes(plan, args, shapes, dtypes, scalars) or [0] * len(args)
    ok, why = _tc_ok(plan, dtypes)
    if ok:
        if variant == "pair" or (variant == "auto" and plan.M >= PAIR_BM and plan.N >= BN):
            ks = _gen_tcgen05_pair(kop, plan, shapes, dtypes, args, ptrs, sig, params, scalar_env, rbytes, tune)
        else:
            ks = _gen_tcgen05(kop, plan, shapes, dtypes, args, ptrs, sig, params, scalar_env, rbytes)
    else:
        ks = _gen_simt(kop, plan, shapes, dtypes, args, ptrs, sig, params, scalar_env, why, rbytes)
    return _with_dropin(ks, kop, plan, shapes, dtypes, ptrs, sig, scalar_env, meta_threads)


def _with_dropin(ks: KernelSource, kop, plan: GemmPlan, shapes, dtypes, ptrs, sig, scalar_env,
                 meta_threads: int) -> KernelSource:
    """Rename the fast kernel to ``<name>__emmy`` (the entry libemmy_b200
    launches, with tensor maps and a row range after the buffers) and add the
    drop-in ``<name>``: ``arg_order`` parameters only, correct under any
    launch.  It tiles C in shared memory and runs every output as one
    sequential ``fma.rn`` chain over k, in f32 (bf16/f16 operands are widened
    exactly), so its results equal the reference's f32 route bit for bit."""
    from .dropin import _header, native_entry
    m = _header(ks.source, kop.name)
    hdr = ks.source[m.start():m.end()].replace(f" {kop.name}(", f" {native_entry(kop.name)}(", 1)
    src = ks.source[:m.start()] + hdr + ks.source[m.end():]
    src += "\n" + _dropin_source(kop, plan, shapes, dtypes, ptrs, sig, scalar_env, meta_threads)
    notes = dict(ks.notes)
    notes["entries"] = {"drop_in": kop.name, "native": native_entry(kop.name),
                        "drop_in_path": "shared-memory tiled exact-order f32 GEMM, any launch"}
    return KernelSource(entry=ks.entry, source=src, launch=ks.launch, params=ks.params, family=ks.family,
                        notes=notes, tmaps=ks.tmaps)


def _dropin_source(kop, plan: GemmPlan, shapes, dtypes, ptrs, sig, scalar_env, meta_threads: int) -> str:
    M, N, K = plan.M, plan.N, plan.K
    adt = plan.ab_dtype
    a_ptr, b_ptr = ptrs[plan.a.input], ptrs[plan.b.input]
    conv = {"f32": "{x}", "bf16": "__bfloat162float({x})", "f16": "__half2float({x})"}[adt]
    b_elem = (f"{b_ptr}[(long long)gn * K + gk]" if plan.b_nk else f"{b_ptr}[(long long)gk * N + gn]")
    epi = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "acc[ii][jj]", "gi", "gj", " " * 20, None)
    epi1 = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "acc1", "gi", "gj", " " * 8, None)
    seed = f32_lit(plan.seed)
    cname = _c(kop.name)
    names = ", ".join(s.split()[-1] for s in sig)
    lb = max(256, meta_threads or 0)
    return f"""
namespace {{
constexpr long long DM_M = {M}LL, DM_N = {N}LL, DM_K = {K}LL;

// one CTA-tile of TBM x TBN outputs at a time, grid-stride over tiles; the
// (TBM/4) x (TBN/4) worker threads each own a 4 x 4 block of outputs
template <int TBM, int TBN>
__device__ __forceinline__ void emmy_dropin_tiles_{cname}({", ".join(sig)}, int tid, int nthr) {{
    constexpr long long M = DM_M, N = DM_N, K = DM_K;
    constexpr int TBK = 16, TX = TBN / 4, T = (TBM / 4) * TX;
    __shared__ float sa[TBK][TBM + 1];
    __shared__ float sb[TBK][TBN + 1];
    const long long MB = (M + TBM - 1) / TBM, NB = (N + TBN - 1) / TBN;
    const long long cta = (long long)blockIdx.x + (long long)gridDim.x * (blockIdx.y + (long long)gridDim.y * blockIdx.z);
    const long long ncta = (long long)gridDim.x * gridDim.y * gridDim.z;
    const bool worker = tid < T;
    const int tx = tid % TX, ty = tid / TX;
    for (long long t = cta; t < MB * NB; t += ncta) {{
        const long long m0 = (t / NB) * TBM, n0 = (t % NB) * TBN;
        float acc[4][4];
        #pragma unroll
        for (int a = 0; a < 4; ++a)
            #pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = {seed};
        for (long long k0 = 0; k0 < K; k0 += TBK) {{
            for (int e = tid; e < TBK * TBM; e += nthr) {{
                const int kk = e % TBK, mm = e / TBK;
                const long long gm = m0 + mm, gk = k0 + kk;
                sa[kk][mm] = (gm < M && gk < K) ? {conv.format(x=f"{a_ptr}[gm * K + gk]")} : 0.0f;
            }}
            for (int e = tid; e < TBK * TBN; e += nthr) {{
                const int kk = e / TBN, nn = e % TBN;
                const long long gn = n0 + nn, gk = k0 + kk;
                sb[kk][nn] = (gn < N && gk < K) ? {conv.format(x=b_elem)} : 0.0f;
            }}
            __syncthreads();
            if (worker) {{
                const int kmax = (K - k0) < TBK ? (int)(K - k0) : TBK;
                for (int kk = 0; kk < kmax; ++kk) {{
                    float av[4], bv[4];
                    #pragma unroll
                    for (int a = 0; a < 4; ++a) av[a] = sa[kk][ty * 4 + a];
                    #pragma unroll
                    for (int b = 0; b < 4; ++b) bv[b] = sb[kk][tx * 4 + b];
                    #pragma unroll
                    for (int a = 0; a < 4; ++a)
                        #pragma unroll
                        for (int b = 0; b < 4; ++b) acc[a][b] = __fmaf_rn(av[a], bv[b], acc[a][b]);
                }}
            }}
            __syncthreads();
        }}
        if (worker) {{
            #pragma unroll
            for (int ii = 0; ii < 4; ++ii) {{
                #pragma unroll
                for (int jj = 0; jj < 4; ++jj) {{
                    const long long gi = m0 + ty * 4 + ii, gj = n0 + tx * 4 + jj;
                    if (gi < M && gj < N) {{
{chr(10).join(epi)}
                    }}
                }}
            }}
        }}
    }}
}}
}}  // namespace

extern "C" __global__ void __launch_bounds__({lb}) {kop.name}({", ".join(sig)}) {{
    const int nthr = (int)(blockDim.x * blockDim.y * blockDim.z);
    const int tid = (int)((threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x);
    if (nthr >= 256) {{ emmy_dropin_tiles_{cname}<64, 64>({names}, tid, nthr); return; }}
    if (nthr >= 128) {{ emmy_dropin_tiles_{cname}<32, 64>({names}, tid, nthr); return; }}
    if (nthr >= 64) {{ emmy_dropin_tiles_{cname}<32, 32>({names}, tid, nthr); return; }}
    if (nthr >= 32) {{ emmy_dropin_tiles_{cname}<16, 32>({names}, tid, nthr); return; }}
    // fewer than 32 threads per block: one output per thread
    constexpr long long M = DM_M, N = DM_N, K = DM_K;
    const long long gstride = (long long)gridDim.x * gridDim.y * gridDim.z * nthr;
    const long long cta = (long long)blockIdx.x + (long long)gridDim.x * (blockIdx.y + (long long)gridDim.y * blockIdx.z);
    for (long long o = cta * nthr + tid; o < M * N; o += gstride) {{
        const long long gi = o / N, gj = o % N;
        float acc1 = {seed};
        for (long long gk = 0; gk < K; ++gk) {{
            const long long gm = gi, gn = gj;
            acc1 = __fmaf_rn({conv.format(x=f"{a_ptr}[gm * K + gk]")}, {conv.format(x=b_elem)}, acc1);
        }}
{chr(10).join(epi1)}
    }}
}}
"""


# ---------------------------------------------------------------------------- epilogue


def _epilogue_code(plan: GemmPlan, shapes, dtypes, ptrs, scalar_env, acc_code: str, i_code: str,
                   j_code: str, ind: str, out_var: str | None) -> list[str]:
    """The IR's post-loop statements for one output, with the accumulator
    bound to ``acc_code``.  With ``out_var`` the C write is captured into that
    variable (converted to C's element type) instead of stored."""

    def write_hook(s, k, kind, code):
        dt = ir.canon_dtype(s.value_dtype or dtypes.get(s.output))
        if out_var is not None and s is plan.out:
            return f"{out_var} = {store_from(kind, code, dt)};"
        return em._default_write(s, k, kind, code)

    em = Emitter(shapes, dtypes, ptrs, write_hook=write_hook, indent=ind)
    em.env.update(scalar_env)
    em.bind_const(plan.i, "int", i_code)
    em.bind_const(plan.j, "int", j_code)
    em.assign(plan.acc, "f32", acc_code)
    em.run(plan.epilogue)
    return em.lines


# ---------------------------------------------------------------------------- tcgen05


def _gen_tcgen05(kop, plan: GemmPlan, shapes, dtypes, args, ptrs, sig, params, scalar_env,
                 rbytes) -> KernelSource:
    M, N, K = plan.M, plan.N, plan.K
    mb, nb, kb = -(-M // BM), -(-N // BN), -(-K // BK)
    tiles = mb * nb
    odt = ir.canon_dtype(plan.out.value_dtype or dtypes.get(plan.out.output))
    ocls = ctype(odt)
    fmt = 1 if plan.ab_dtype == "bf16" else 0
    a_idx = args.index(plan.a.input)
    b_idx = args.index(plan.b.input)
    esz = 2
    tm_a = TmapSpec(a_idx, TMAP_DTYPE[plan.ab_dtype], [K, M], [K * esz], [BK, BM], SWIZZLE_128B, L2_256B)
    if plan.b_nk:
        tm_b = TmapSpec(b_idx, TMAP_DTYPE[plan.ab_dtype], [K, N], [K * esz], [BK, BN], SWIZZLE_128B, L2_256B)
    else:
        tm_b = TmapSpec(b_idx, TMAP_DTYPE[plan.ab_dtype], [N, K], [N * esz], [64, BK], SWIZZLE_128B, L2_256B)
    a_stage = BM * BK * esz
    b_stage = BN * BK * esz
    smem = 1024 + STAGES * (a_stage + b_stage) + 256
    sig = list(sig) + ["const __grid_constant__ CUtensorMap tm_a", "const __grid_constant__ CUtensorMap tm_b"] + RANGE_SIG
    out_ptr = ptrs[plan.out.output]
    vec_store = (N % 8 == 0) if odt in ("bf16", "f16") else (N % 4 == 0)
    epi_full = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "__uint_as_float(r[jj])", "row",
                              "(col0 + jj)", " " * 24, "ov[jj]")
    epi_any = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "__uint_as_float(r[jj])", "row",
                             "(col0 + jj)", " " * 28, "ov1")
    if odt in ("bf16", "f16"):
        pack = ("                    uint4 *dst = reinterpret_cast<uint4 *>(" + out_ptr + " + row * (long long)N + col0);\n"
                "                    #pragma unroll\n"
                "                    for (int v = 0; v < 4; ++v) {\n"
                "                        uint4 w;\n"
                "                        memcpy(&w, &ov[v * 8], 16);\n"
                "                        dst[v] = w;\n"
                "                    }\n")
    else:
        pack = ("                    float4 *dst = reinterpret_cast<float4 *>(" + out_ptr + " + row * (long long)N + col0);\n"
                "                    #pragma unroll\n"
                "                    for (int v = 0; v < 8; ++v) dst[v] = make_float4(ov[4*v], ov[4*v+1], ov[4*v+2], ov[4*v+3]);\n")
    src = f"""{DEVICE_PRELUDE}
#include <string.h>
#include "emmy_sm100.cuh"

namespace {{
constexpr long long M = {M}LL, N = {N}LL, K = {K}LL;
constexpr int BM = {BM}, BN = {BN}, BK = {BK}, STAGES = {STAGES};
constexpr int NB = {nb}, KB = {kb}, GROUP_M = {GROUP_M};
constexpr uint32_t A_STAGE = {a_stage}u, B_STAGE = {b_stage}u;
constexpr uint32_t SMEM_BYTES = {smem}u;
constexpr uint32_t IDESC = emmy::idesc_f16({fmt}u, {0 if plan.b_nk else 1}u, BM, BN);
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s per wait: orders of magnitude above any legal wait

// tile t of a launch over row-tiles [mb0, mb0 + mbn): GROUP_M row-tiles share each column sweep
__device__ __forceinline__ void tile_coords(int t, int mb0, int mbn, int &mb, int &nb) {{
    const int per_group = GROUP_M * NB;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int first = g * GROUP_M;
    const int rows = (mbn - first) < GROUP_M ? (mbn - first) : GROUP_M;
    mb = mb0 + first + r % rows;
    nb = r / rows;
}}
}}  // namespace

extern "C" __global__ void __launch_bounds__({TC_THREADS}, 1) {kop.name}({", ".join(sig)}) {{
{_row_range(BM, mb)}    uint32_t dyn_smem;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));
    if (blockDim.x != {TC_THREADS} || blockDim.y != 1 || blockDim.z != 1 || dyn_smem < SMEM_BYTES) {{
        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);
        return;
    }}
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_STAGE;
    uint64_t *full = reinterpret_cast<uint64_t *>(sB + STAGES * B_STAGE);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_holder + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {{
        for (int s = 0; s < STAGES; ++s) {{ emmy::mbar_init(&full[s], 1); emmy::mbar_init(&empty[s], 1); }}
        for (int a = 0; a < 2; ++a) {{ emmy::mbar_init(&tfull[a], 1); emmy::mbar_init(&tempty[a], 4); }}
        emmy::mbar_init(drain, 1);
        *abort_flag = 0u;
        emmy::fence_barrier_init();
    }}
    if (warp == 1) {{
        emmy::tmem_alloc(tmem_holder, 512);
        emmy::tmem_relinquish();
    }}
    if (warp == 0 && lane == 0) {{
        emmy::tma_prefetch(&tm_a);
        emmy::tma_prefetch(&tm_b);
    }}
    emmy::tc_fence_before();
    __syncthreads();
    emmy::tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {{
        if (lane == 0) {{
            // ---------------- TMA producer
            uint32_t stage = 0, phase = 0;
            uint32_t issued = 0u, parity_bits = 0u;  // per stage: load in flight, its phase parity
            bool ok = true;
            for (int t = blockIdx.x; t < TILES && ok; t += gridDim.x) {{
                int tm, tn;
                tile_coords(t, MB0, MBN, tm, tn);
                for (int k = 0; k < KB; ++k) {{
                    if (!emmy::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, EMMY_STATUS_TIMEOUT_PRODUCER, WAIT_NS)) {{ ok = false; break; }}
                    emmy::mbar_arrive_expect_tx(&full[stage], A_STAGE + B_STAGE);
                    emmy::tma_load_2d(sA + stage * A_STAGE, &tm_a, &full[stage], k * BK, (tm - MB0) * BM);
{_b_loads(plan.b_nk)}
                    issued |= 1u << stage;
                    parity_bits = (parity_bits & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {{ stage = 0; phase ^= 1u; }}
                }}
            }}
            if (!ok) {{
                // drain this CTA's own loads still in flight before teardown (bounded)
                volatile uint32_t never = 0u;
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s)) emmy::mbar_wait(&full[s], (parity_bits >> s) & 1u, &never, 0u, 20000000ull);
            }}
        }}
        __syncwarp();
    }} else if (warp == 1) {{
        if (lane == 0) {{
            // ---------------- MMA issuer
            uint32_t stage = 0, phase = 0, it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < TILES && ok; t += gridDim.x, ++it) {{
                const uint32_t acc = it & 1u, aphase = (it >> 1) & 1u;
                if (!emmy::mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) break;
                emmy::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int k = 0; k < KB; ++k) {{
                    if (!emmy::mbar_wait(&full[stage], phase, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) {{ ok = false; break; }}
                    emmy::tc_fence_after();
                    const uint32_t a_base = emmy::smem_u32(sA + stage * A_STAGE);
                    const uint32_t b_base = emmy::smem_u32(sB + stage * B_STAGE);
                    #pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {{
                        const uint64_t ad = emmy::smem_desc_sw128(a_base + kk * 32, 16, 1024);
{_b_desc(plan.b_nk)}
                        emmy::umma_f16(d_tmem, ad, bd, IDESC, (k | kk) != 0 ? 1u : 0u);
                    }}
                    emmy::umma_commit(&empty[stage]);
                    if (++stage == STAGES) {{ stage = 0; phase ^= 1u; }}
                }}
                if (!ok) break;
                emmy::umma_commit(&tfull[acc]);
            }}
            // every MMA this thread issued has finished before TMEM is released (bounded)
            emmy::umma_commit(drain);
            volatile uint32_t never = 0u;
            emmy::mbar_wait(drain, 0u, &never, 0u, 20000000ull);
        }}
        __syncwarp();
    }} else {{
        // ---------------- epilogue: TMEM -> registers -> IR epilogue -> C
        const int q = warp & 3;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < TILES; t += gridDim.x, ++it) {{
            const uint32_t acc = it & 1u, aphase = (it >> 1) & 1u;
            if (!emmy::mbar_wait(&tfull[acc], aphase, abort_flag, EMMY_STATUS_TIMEOUT_EPILOGUE, WAIT_NS)) break;
            emmy::tc_fence_after();
            int tm, tn;
            tile_coords(t, MB0, MBN, tm, tn);
            const long long row = (long long)tm * BM + q * 32 + lane;
            #pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {{
                uint32_t r[32];
                emmy::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, r);
                emmy::tmem_ld_wait();
                const long long col0 = (long long)tn * BN + c * 32;
                if (row < M && col0 + 32 <= N && {'true' if vec_store else 'false'}) {{
                    {ocls} ov[32];
                    #pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {{
{chr(10).join(epi_full)}
                    }}
{pack}                }} else if (row < M) {{
                    #pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {{
                        if (col0 + jj < N) {{
                            {ocls} ov1;
{chr(10).join(epi_any)}
                            {out_ptr}[row * N + col0 + jj] = ov1;
                        }}
                    }}
                }}
            }}
            emmy::tc_fence_before();
            __syncwarp();
            if (lane == 0) emmy::mbar_arrive(&tempty[acc]);
        }}
    }}
    emmy::tc_fence_before();
    __syncthreads();
    if (warp == 1) {{
        emmy::tc_fence_after();
        emmy::tmem_dealloc(tmem_base, 512);
    }}
}}
"""
    grid = max(1, min(tiles, SM_COUNT))
    launch = LaunchPlan(grid=(grid, 1, 1), block=(TC_THREADS, 1, 1), smem=smem,
                        range_total=M, range_align=BM, range_bytes=rbytes)
    src += launch_record_source("gemm", launch, params, [tm_a, tm_b])
    notes = {"kernel": "tcgen05", "tile": [BM, BN, BK], "stages": STAGES, "tiles": tiles,
             "b_layout": "NK" if plan.b_nk else "KN", "vector_store": vec_store}
    return KernelSource(entry=kop.name, source=src, launch=launch, params=params, family="gemm",
                        notes=notes, tmaps=[tm_a, tm_b])


def _b_loads(b_nk: bool) -> str:
    ind = " " * 20
    if b_nk:
        return f"{ind}emmy::tma_load_2d(sB + stage * B_STAGE, &tm_b, &full[stage], k * BK, tn * BN);"
    return "\n".join(
        f"{ind}emmy::tma_load_2d(sB + stage * B_STAGE + {j * 8192}u, &tm_b, &full[stage], tn * BN + {64 * j}, k * BK);"
        for j in range(BN // 64))


def _b_desc(b_nk: bool) -> str:
    ind = " " * 24
    if b_nk:
        return f"{ind}const uint64_t bd = emmy::smem_desc_sw128(b_base + kk * 32, 16, 1024);"
    # MN-major: 64-column blocks 8 KB apart (LBO), 8-row K groups 1 KB apart (SBO); 16 K rows = 2 KB
    return f"{ind}const uint64_t bd = emmy::smem_desc_sw128(b_base + kk * 2048, 8192, 1024);"


# ---------------------------------------------------------------------------- SIMT


def _gen_simt(kop, plan: GemmPlan, shapes, dtypes, args, ptrs, sig, params, scalar_env, why,
              rbytes) -> KernelSource:
    M, N, K = plan.M, plan.N, plan.K
    mb, nb = -(-M // SIMT_BM), -(-N // SIMT_BN)
    tiles = mb * nb
    adt = plan.ab_dtype
    a_ptr, b_ptr = ptrs[plan.a.input], ptrs[plan.b.input]
    conv = {"f32": "{x}", "bf16": "__bfloat162float({x})", "f16": "__half2float({x})"}[adt]
    b_elem = (f"{b_ptr}[(long long)gn * K + gk]" if plan.b_nk else f"{b_ptr}[(long long)gk * N + gn]")
    epi = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "acc[ii][jj]", "gi", "gj", " " * 16, None)
    seed = f32_lit(plan.seed)
    src = f"""{DEVICE_PRELUDE}
#include "emmy_launch_record.h"
extern "C" __device__ unsigned int emmy_status;

extern "C" __global__ void __launch_bounds__({SIMT_THREADS}) {kop.name}({", ".join(sig + RANGE_SIG)}) {{
    constexpr long long M = {M}LL, N = {N}LL, K = {K}LL;
    constexpr int TBM = {SIMT_BM}, TBN = {SIMT_BN}, TBK = {SIMT_BK}, NB = {nb};
{_row_range(SIMT_BM, mb)}
    if (blockDim.x != {SIMT_THREADS} || blockDim.y != 1 || blockDim.z != 1) {{
        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);
        return;
    }}
    __shared__ float sa[TBK][TBM + 1];
    __shared__ float sb[TBK][TBN + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    for (int t = blockIdx.x; t < TILES; t += gridDim.x) {{
        const long long m0 = (long long)(MB0 + t / NB) * TBM, n0 = (long long)(t % NB) * TBN;
        float acc[4][4];
        #pragma unroll
        for (int a = 0; a < 4; ++a)
            #pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = {seed};
        for (long long k0 = 0; k0 < K; k0 += TBK) {{
            for (int e = threadIdx.x; e < TBK * TBM; e += blockDim.x) {{
                const int kk = e % TBK, mm = e / TBK;
                const long long gm = m0 + mm, gk = k0 + kk;
                sa[kk][mm] = (gm < M && gk < K) ? {conv.format(x=f"{a_ptr}[gm * K + gk]")} : 0.0f;
            }}
            for (int e = threadIdx.x; e < TBK * TBN; e += blockDim.x) {{
                const int kk = e / TBN, nn = e % TBN;
                const long long gn = n0 + nn, gk = k0 + kk;
                sb[kk][nn] = (gn < N && gk < K) ? {conv.format(x=b_elem)} : 0.0f;
            }}
            __syncthreads();
            const int kmax = (K - k0) < TBK ? (int)(K - k0) : TBK;
            for (int kk = 0; kk < kmax; ++kk) {{
                float av[4], bv[4];
                #pragma unroll
                for (int a = 0; a < 4; ++a) av[a] = sa[kk][ty * 4 + a];
                #pragma unroll
                for (int b = 0; b < 4; ++b) bv[b] = sb[kk][tx * 4 + b];
                #pragma unroll
                for (int a = 0; a < 4; ++a)
                    #pragma unroll
                    for (int b = 0; b < 4; ++b) acc[a][b] = __fmaf_rn(av[a], bv[b], acc[a][b]);
            }}
            __syncthreads();
        }}
        #pragma unroll
        for (int ii = 0; ii < 4; ++ii) {{
            #pragma unroll
            for (int jj = 0; jj < 4; ++jj) {{
                const long long gi = m0 + ty * 4 + ii, gj = n0 + tx * 4 + jj;
                if (gi < M && gj < N) {{
{chr(10).join(epi)}
                }}
            }}
        }}
    }}
}}
"""
    grid = max(1, min(tiles, SM_COUNT * 8))
    launch = LaunchPlan(grid=(grid, 1, 1), block=(SIMT_THREADS, 1, 1), smem=0,
                        range_total=M, range_align=SIMT_BM, range_bytes=rbytes)
    src += launch_record_source("gemm", launch, params)
    notes = {"kernel": "simt", "tile": [SIMT_BM, SIMT_BN, SIMT_BK], "tiles": tiles, "why_not_tcgen05": why}
    return KernelSource(entry=kop.name, source=src, launch=launch, params=params, family="gemm", notes=notes)


# ---------------------------------------------------------------------------- tcgen05, CTA pair


def _gen_tcgen05_pair(kop, plan: GemmPlan, shapes, dtypes, args, ptrs, sig, params, scalar_env,
                      rbytes, tune: dict | None = None) -> KernelSource:
    """256x256 tiles on a cluster of two CTAs (``cta_group::2``): each CTA loads
    its 128 rows of A and its 128 columns of B per stage (32 KB instead of the
    single-CTA kernel's 48 KB for half the FLOPs), the leader issues
    ``tcgen05.mma.cta_group::2`` 256x256x16 over both CTAs' shared memory into
    both CTAs' tensor memory, and each CTA's epilogue drains its own 128 rows.
    6 pipeline stages fit in shared memory."""
    tn_ = {**PAIR_TUNE, **(tune or {})}
    M, N, K = plan.M, plan.N, plan.K
    mb, nb, kb = -(-M // PAIR_BM), -(-N // BN), -(-K // BK)
    tiles = mb * nb
    odt = ir.canon_dtype(plan.out.value_dtype or dtypes.get(plan.out.output))
    ocls = ctype(odt)
    fmt = 1 if plan.ab_dtype == "bf16" else 0
    a_idx, b_idx = args.index(plan.a.input), args.index(plan.b.input)
    esz = 2
    cbm, cbn = PAIR_BM // 2, BN // 2
    tm_a = TmapSpec(a_idx, TMAP_DTYPE[plan.ab_dtype], [K, M], [K * esz], [BK, cbm], SWIZZLE_128B, L2_256B)
    if plan.b_nk:
        tm_b = TmapSpec(b_idx, TMAP_DTYPE[plan.ab_dtype], [K, N], [K * esz], [BK, cbn], SWIZZLE_128B, L2_256B)
    else:
        tm_b = TmapSpec(b_idx, TMAP_DTYPE[plan.ab_dtype], [N, K], [N * esz], [64, BK], SWIZZLE_128B, L2_256B)
    a_stage = cbm * BK * esz
    b_stage = cbn * BK * esz
    smem = 1024 + PAIR_STAGES * (a_stage + b_stage) + 256
    sig = list(sig) + ["const __grid_constant__ CUtensorMap tm_a", "const __grid_constant__ CUtensorMap tm_b"] + RANGE_SIG
    out_ptr = ptrs[plan.out.output]
    vec_store = (N % 8 == 0) if odt in ("bf16", "f16") else (N % 4 == 0)
    epi_full = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "__uint_as_float(r[jj])", "row",
                              "(col0 + jj)", " " * 24, "ov[jj]")
    epi_any = _epilogue_code(plan, shapes, dtypes, ptrs, scalar_env, "__uint_as_float(r[jj])", "row",
                             "(col0 + jj)", " " * 28, "ov1")
    if odt in ("bf16", "f16"):
        pack = ("                    uint4 *dst = reinterpret_cast<uint4 *>(" + out_ptr + " + row * (long long)N + col0);\n"
                "                    #pragma unroll\n"
                "                    for (int v = 0; v < 4; ++v) {\n"
                "                        uint4 w;\n"
                "                        memcpy(&w, &ov[v * 8], 16);\n"
                "                        " + ("__stcs(&dst[v], w);" if tn_["c_store"] == "cs" else "dst[v] = w;") + "\n"
                "                    }\n")
    else:
        pack = ("                    float4 *dst = reinterpret_cast<float4 *>(" + out_ptr + " + row * (long long)N + col0);\n"
                "                    #pragma unroll\n"
                "                    for (int v = 0; v < 8; ++v) dst[v] = make_float4(ov[4*v], ov[4*v+1], ov[4*v+2], ov[4*v+3]);\n")
    bpol = "pol_b" if tn_["b_policy"] else None
    apol = "pol_a" if tn_["a_policy"] else None

    def _ld(call_args: str, pol) -> str:
        return (f"emmy::tma_load_2d_pair({call_args});" if pol is None
                else f"emmy::tma_load_2d_pair_hint({call_args}, {pol});")

    policies = "".join(
        f"            const uint64_t {var} = emmy::l2_policy_{tn_[key].replace('evict_', 'evict_')}();\n"
        for var, key in (("pol_a", "a_policy"), ("pol_b", "b_policy")) if tn_[key])
    # A's tensor map starts at this launch's first row (the loader encodes it per unit range)
    a_load = "                    " + _ld("sA + stage * A_STAGE, &tm_a, fbar, k * BK, (tm - MB0) * BM + (int)rank * CBM",
                                        apol)
    skip_open = skip_close = ""
    if tn_["skip_first_load"]:
        skip_open = "                    if (!(rank == 1u && pair == 0 && t == pair && k == 0)) {\n"
        skip_close = "\n                    }"
    if plan.b_nk:
        b_loads = "                    " + _ld("sB + stage * B_STAGE, &tm_b, fbar, k * BK, tn * BN + (int)rank * CBN",
                                               bpol)
        b_desc = "                        const uint64_t bd = emmy::smem_desc_sw128(b_base + kk * 32, 16, 1024);"
    else:
        b_loads = "\n".join(
            "                    " + _ld(f"sB + stage * B_STAGE + {j * 8192}u, &tm_b, fbar, "
                                          f"tn * BN + (int)rank * CBN + {64 * j}, k * BK", bpol)
            for j in range(cbn // 64))
        b_desc = "                        const uint64_t bd = emmy::smem_desc_sw128(b_base + kk * 2048, 8192, 1024);"
    src = f"""{DEVICE_PRELUDE}
#include <string.h>
#include "emmy_sm100.cuh"

namespace {{
constexpr long long M = {M}LL, N = {N}LL, K = {K}LL;
constexpr int BM = {PAIR_BM}, CBM = {cbm}, BN = {BN}, CBN = {cbn}, BK = {BK}, STAGES = {PAIR_STAGES};
constexpr int NB = {nb}, KB = {kb}, GROUP_M = {tn_['group_m']};
constexpr uint32_t A_STAGE = {a_stage}u, B_STAGE = {b_stage}u;
constexpr uint32_t SMEM_BYTES = {smem}u;
constexpr uint32_t IDESC = emmy::idesc_f16({fmt}u, {0 if plan.b_nk else 1}u, BM, BN);
constexpr uint64_t WAIT_NS = {int(tn_["wait_ns"])}ull;  // per wait (2 s by default: orders of magnitude above any legal wait)

// tile t of a launch over row-tiles [mb0, mb0 + mbn): GROUP_M row-tiles share each column sweep
__device__ __forceinline__ void tile_coords(int t, int mb0, int mbn, int &mb, int &nb) {{
    const int per_group = GROUP_M * NB;
    const int g = t / per_group;
    const int r = t - g * per_group;
    const int first = g * GROUP_M;
    const int rows = (mbn - first) < GROUP_M ? (mbn - first) : GROUP_M;
    mb = mb0 + first + r % rows;
    nb = r / rows;
}}
}}  // namespace

extern "C" __global__ void __launch_bounds__({TC_THREADS}, 1) {kop.name}({", ".join(sig)}) {{
{_row_range(PAIR_BM, mb)}    uint32_t dyn_smem;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));
    if (blockDim.x != {TC_THREADS} || blockDim.y != 1 || blockDim.z != 1 || dyn_smem < SMEM_BYTES ||
        emmy::cluster_nctarank() != 2u || (gridDim.x & 1u)) {{
        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);
        return;
    }}
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_STAGE;
    uint64_t *full = reinterpret_cast<uint64_t *>(sB + STAGES * B_STAGE);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_holder + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = emmy::cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {{
        for (int s = 0; s < STAGES; ++s) {{ emmy::mbar_init(&full[s], 1); emmy::mbar_init(&empty[s], 1); }}
        for (int a = 0; a < 2; ++a) {{ emmy::mbar_init(&tfull[a], 1); emmy::mbar_init(&tempty[a], 8); }}
        emmy::mbar_init(drain, 1);
        *abort_flag = 0u;
        emmy::fence_barrier_init();
    }}
    if (warp == 1) {{
        emmy::tmem_alloc_pair(tmem_holder, 512);
        emmy::tmem_relinquish_pair();
    }}
    if (warp == 0 && lane == 0) {{
        emmy::tma_prefetch(&tm_a);
        emmy::tma_prefetch(&tm_b);
    }}
    emmy::tc_fence_before();
    __syncthreads();
    emmy::cluster_sync();  // the peer signals the leader's barriers only after both are initialised
    emmy::tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {{
        if (lane == 0) {{
            // ---------------- TMA producer (both CTAs; completion counted on the leader's barrier)
{policies}            uint32_t stage = 0, phase = 0;
            uint32_t issued = 0u, parity_bits = 0u;
            bool ok = true;
            for (int t = pair; t < TILES && ok; t += npairs) {{
                int tm, tn;
                tile_coords(t, MB0, MBN, tm, tn);
                for (int k = 0; k < KB; ++k) {{
                    if (!emmy::mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, EMMY_STATUS_TIMEOUT_PRODUCER, WAIT_NS)) {{ ok = false; break; }}
                    if (rank == 0) emmy::mbar_arrive_expect_tx(&full[stage], 2u * (A_STAGE + B_STAGE));
                    const uint32_t fbar = emmy::mapa(&full[stage], 0);
{skip_open}{a_load}
{b_loads}{skip_close}
                    if (rank == 0) {{
                        issued |= 1u << stage;
                        parity_bits = (parity_bits & ~(1u << stage)) | (phase << stage);
                    }}
                    if (++stage == STAGES) {{ stage = 0; phase ^= 1u; }}
                }}
            }}
            if (!ok && rank == 0) {{
                volatile uint32_t never = 0u;
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s)) emmy::mbar_wait_cluster(&full[s], (parity_bits >> s) & 1u, &never, 0u, 20000000ull);
            }}
        }}
        __syncwarp();
    }} else if (warp == 1) {{
        if (lane == 0) {{
            if (rank == 0) {{
                // ---------------- MMA issuer (leader CTA only)
                uint32_t stage = 0, phase = 0, it = 0;
                bool ok = true;
                const uint32_t peer_empty0 = emmy::mapa(&empty[0], 1);
                for (int t = pair; t < TILES && ok; t += npairs, ++it) {{
                    const uint32_t acc = it & 1u, aphase = (it >> 1) & 1u;
                    if (!emmy::mbar_wait_cluster(&tempty[acc], aphase ^ 1u, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) break;
                    emmy::tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BN;
                    for (int k = 0; k < KB; ++k) {{
                        if (!emmy::mbar_wait_cluster(&full[stage], phase, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) {{ ok = false; break; }}
                        emmy::tc_fence_after();
                        const uint32_t a_base = emmy::smem_u32(sA + stage * A_STAGE);
                        const uint32_t b_base = emmy::smem_u32(sB + stage * B_STAGE);
                        #pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {{
                            const uint64_t ad = emmy::smem_desc_sw128(a_base + kk * 32, 16, 1024);
{b_desc}
                            emmy::umma_f16_pair(d_tmem, ad, bd, IDESC, (k | kk) != 0 ? 1u : 0u);
                        }}
                        emmy::umma_commit_pair(emmy::smem_u32(&empty[stage]));
                        emmy::umma_commit_pair(peer_empty0 + stage * 8u);
                        if (++stage == STAGES) {{ stage = 0; phase ^= 1u; }}
                    }}
                    if (!ok) break;
                    emmy::umma_commit_pair(emmy::smem_u32(&tfull[acc]));
                    emmy::umma_commit_pair(emmy::mapa(&tfull[acc], 1));
                }}
                // arrives on both CTAs once every pair MMA has finished
                emmy::umma_commit_pair(emmy::smem_u32(drain));
                emmy::umma_commit_pair(emmy::mapa(drain, 1));
            }}
        }}
        __syncwarp();
    }} else {{
        // ---------------- epilogue (both CTAs): own 128 rows of the 256x256 tile
        const int q = warp & 3;
        const uint32_t leader_tempty0 = emmy::mapa(&tempty[0], 0);
        uint32_t it = 0;
        for (int t = pair; t < TILES; t += npairs, ++it) {{
            const uint32_t acc = it & 1u, aphase = (it >> 1) & 1u;
            if (!emmy::mbar_wait_cluster(&tfull[acc], aphase, abort_flag, EMMY_STATUS_TIMEOUT_EPILOGUE, WAIT_NS)) break;
            emmy::tc_fence_after();
            int tm, tn;
            tile_coords(t, MB0, MBN, tm, tn);
            const long long row = (long long)tm * BM + (int)rank * CBM + q * 32 + lane;
            #pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {{
                uint32_t r[32];
                emmy::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, r);
                emmy::tmem_ld_wait();
                const long long col0 = (long long)tn * BN + c * 32;
                if (row < M && col0 + 32 <= N && {'true' if vec_store else 'false'}) {{
                    {ocls} ov[32];
                    #pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {{
{chr(10).join(epi_full)}
                    }}
{pack}                }} else if (row < M) {{
                    #pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {{
                        if (col0 + jj < N) {{
                            {ocls} ov1;
{chr(10).join(epi_any)}
                            {out_ptr}[row * N + col0 + jj] = ov1;
                        }}
                    }}
                }}
            }}
            emmy::tc_fence_before();
            __syncwarp();
            if (lane == 0) emmy::mbar_arrive_cluster(leader_tempty0 + acc * 8u);
        }}
    }}
    emmy::tc_fence_before();
    __syncthreads();
    if (warp == 1) {{
        // the last MMA, and the leader's last commit into this CTA, have landed (bounded)
        if (lane == 0) {{
            volatile uint32_t never = 0u;
            emmy::mbar_wait_cluster(drain, 0u, &never, 0u, WAIT_NS);
        }}
        __syncwarp();
    }}
    emmy::cluster_sync();  // no CTA leaves while its peer may still signal or read it
    if (warp == 1) {{
        emmy::tc_fence_after();
        emmy::tmem_dealloc_pair(tmem_base, 512);
    }}
}}
"""
    grid = max(2, min(tiles * 2, SM_COUNT) // 2 * 2)
    launch = LaunchPlan(grid=(grid, 1, 1), block=(TC_THREADS, 1, 1), smem=smem, cluster=(2, 1, 1),
                        range_total=M, range_align=PAIR_BM, range_bytes=rbytes)
    src += launch_record_source("gemm", launch, params, [tm_a, tm_b])
    notes = {"kernel": "tcgen05_pair", "tile": [PAIR_BM, BN, BK], "stages": PAIR_STAGES, "tiles": tiles,
             "b_layout": "NK" if plan.b_nk else "KN", "vector_store": vec_store, "cluster": 2}
    return KernelSource(entry=kop.name, source=src, launch=launch, params=params, family="gemm",
                        notes=notes, tmaps=[tm_a, tm_b])
