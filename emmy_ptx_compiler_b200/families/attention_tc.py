"""Attention on the 5th-generation tensor cores: the naive attention IR
(tools/make_proxy_set.py:416-490 shape) as one tcgen05 kernel.

Both contractions of the IR run on ``tcgen05.mma.kind::tf32`` with a
three-term split of every f32 operand (``x = hi + lo``, ``hi`` = x with its
13 low mantissa bits cleared, ``lo = x - hi`` exactly; a product is taken as
``hi*hi + hi*lo + lo*hi``), which keeps about 21 bits of each product and
accumulates in f32 in tensor memory:

* scores ``S = q kᵀ`` (M = 128 query rows x N = the CTA's keys, K = head
  size) once per (row, key), kept in tensor memory for every pass of the IR;
* the weighted sum ``O = P v`` (M = 128 rows x N = head size, K = keys), with
  ``P`` the per-(row, key) weight the IR's last key loop computes.

Everything between - the IR's per-key statements (scale, ``exp``, the
weights), its per-row statements (reciprocal of the denominator) and its row
accumulations (max, sum) - runs on CUDA cores with the reference's op table
(cgen), one thread per query row reading its scores from tensor memory.

A query tile of 128 rows is shared by CL CTAs that split the keys: each CTA
computes its keys' scores and partial row statistics, the CTAs exchange the
partials after every key loop (combined in CTA order, so every CTA holds the
same row values), each CTA multiplies its own keys' weights into a partial
``O``, and the partial outputs are added in CTA order, each CTA writing
128 / CL rows.  The exchange goes through distributed shared memory when the
CL CTAs form a cluster, or through global memory with a counter barrier per
tile when every CTA of the problem is resident at once under a cooperative
launch (``layout``'s ``exchange``).

Shared-memory operands use the 128-byte swizzled K-major layout (rows of 32
f32 words, 16-byte chunk c of row r stored at chunk c ^ (r & 7)); all
operands are read from this GPU's memory with ordinary loads.  Every
mbarrier wait is bounded.  Results follow the reference's arithmetic except
for the summation order and the tensor-core products, within rtol 1e-4.
"""

from __future__ import annotations

from .. import ir
from ..cgen import DEVICE_PRELUDE, Emitter, combine_code, ctype, f32_lit, fusable_products, identity_of
from ..errors import UnsupportedIR
from .common import KernelSource, LaunchPlan, ParamSpec, SM_COUNT, launch_record_source
from .common import c_ident as _c

T = 512                 # threads: 4 column groups x 128 query rows of the tile
NG = T // 128           # column groups: warp w reads tensor-memory lanes 32 (w % 4).. and keys group w / 4
SMEM_MAX = 220 * 1024   # dynamic shared memory budget per CTA
TMEM_COLS_MAX = 512
SM_SMEM_BYTES = 228 * 1024   # shared memory of one SM (each resident CTA also takes 1 KB)
# clusters of CL CTAs (one CTA per SM) a B200 holds at once (ncu launch__cluster_max_active: 15
# for clusters of 8); sizes not listed are taken to fit whenever their CTAs do
CLUSTERS_RESIDENT = {8: 15}


def _pad(x: int, m: int) -> int:
    return -(-x // m) * m


def _dep_pattern(st, plan) -> str | None:
    """The weight name ``w`` when the key loop's j-dependent statements are
    exactly ``vv = v[k, j]; p = w * vv; acc += p`` (a matrix product)."""
    dep = list(st.dep)
    if len(dep) != 3:
        return None
    ld, mul, acc = dep
    if not (isinstance(ld, ir.Load) and isinstance(mul, ir.Assign) and isinstance(acc, ir.Accum)):
        return None
    if ld.input != plan.v or len(ld.names) != 1:
        return None
    if ir.op_name(mul.op) not in ("multiply", "mul") or len(mul.args) != 2 or ld.names[0] not in mul.args:
        return None
    if ir.op_name(acc.op) not in ("add", "sum") or acc.value != mul.name or acc.name not in plan.cell_accs:
        return None
    w = mul.args[0] if mul.args[1] == ld.names[0] else mul.args[1]
    if w == ld.names[0] or w not in st.stash:
        return None
    return w


def layout(plan, shapes: dict, dtypes: dict, exchange: str = "auto") -> tuple[dict | None, list[str]]:
    """Tile sizes of the tensor-core kernel for ``plan``, or None with reasons.

    ``exchange``: how the CL CTAs of one query tile combine row values and
    partial outputs.  "cluster": the CTAs form a thread-block cluster and read
    one another's shared memory.  "grid": plain CTAs under a cooperative launch
    (all resident at once) that exchange through global memory behind an
    arrival-counter barrier per tile.  A cluster of 8 CTAs of about 200 KB of shared
    memory needs 8 free SMs of one GPC, so a B200 holds 15 such clusters at
    once: 16 query tiles then run in two rounds, while 128 plain CTAs all fit
    on its 148 SMs.  "auto" takes "grid" when every CTA fits on the SMs at
    once and the clusters would not (``CLUSTERS_RESIDENT``), else "cluster":
    where both fit, the cluster exchange is the faster (a_attn 256 x 64: 17
    against 23 us; 2048 x 64: 58 against 40 us the other way)."""
    from .attention import KeyLoop
    why: list[str] = []
    SQ, SK, D, DV = plan.SQ, plan.SK, plan.D, plan.DV
    keyloops = [s for s in plan.steps if isinstance(s, KeyLoop)]
    if plan.v is None or not keyloops:
        why.append("no weighted sum of v")
        return None, why
    last = keyloops[-1]
    if any(s.dep for s in keyloops[:-1]):
        why.append("j-dependent statements before the last key loop")
    w = _dep_pattern(last, plan) if last.dep else None
    if w is None:
        why.append("last key loop is not acc += w(i, k) * v[k, j]")
    if plan.steps[-1] is not last:
        why.append("row statements after the last key loop")
    if any(s.dot_init != 0.0 for s in keyloops):
        why.append("dot product seeded with a non-zero value")
    if len(plan.cell_accs) != 1 or plan.out.values[0] != plan.cell_accs[0]:
        why.append("output is not the single cell accumulator")
    # the cell accumulator starts at 0 (a row statement Init before the last loop)
    for st in plan.steps:
        if not isinstance(st, KeyLoop) and isinstance(st[1], ir.Init) and st[1].name in plan.cell_accs:
            if float(st[1].identity) != 0.0:
                why.append("cell accumulator seeded with a non-zero value")
    for s in keyloops:
        for a, op in s.row_accs:
            if op not in ("add", "maximum", "minimum"):
                why.append(f"row accumulation {op}")
    if D % 4 or DV % 4:
        why.append("head sizes not multiples of 4")
    if SQ < 64 or SK < 32:
        why.append("fewer than 64 query rows or 32 keys")
    if _pad(DV, 32) > 32 * NG:
        why.append(f"head size {DV} above {32 * NG}")
    if why:
        return None, why
    DP, DVP = _pad(D, 32), _pad(DV, 16)
    nq = -(-SQ // 128)
    best = None
    for CL in (1, 2, 4, 8):
        KC = _pad(-(-SK // CL), 32)
        if CL > 1 and (CL - 1) * KC >= SK:
            continue                   # a CTA without keys
        tcols = 32
        while tcols < KC + _pad(DVP, 32):
            tcols *= 2
        if KC > 256 or tcols > TMEM_COLS_MAX:
            continue
        r1 = max(2 * (DP // 32) * 128 * 128, 4 * 128 * 128, 128 * DVP * 4)
        r2 = max(2 * (DP // 32) * KC * 128, 2 * (KC // 32) * DVP * 128)
        # per accumulator: the cluster exchange slot and the column groups' partials, 128 rows each
        nstat = sum(len(s.row_accs) for s in keyloops) * 128 * 4 * (1 + NG)
        smem = 1024 + r1 + r2 + nstat + 64      # 6 mbarriers, the tensor-memory address, 2 flags
        if smem > SMEM_MAX:
            continue
        cand = dict(CL=CL, KC=KC, DP=DP, DVP=DVP, TCOLS=tcols, R1=r1, R2=r2, NSTAT=nstat, SMEM=smem, nq=nq, W=w)
        best = cand
        if nq * CL >= SM_COUNT // 2:
            break
    if best is None:
        why.append("no cluster split fits shared and tensor memory")
        return best, why
    fits = best["CL"] > 1 and best["nq"] * best["CL"] <= SM_COUNT
    if exchange == "grid" and not fits:
        why.append(f"{best['nq'] * best['CL']} CTAs do not fit on the SMs at once (grid exchange)")
        return None, why
    if exchange not in ("auto", "grid", "cluster"):
        raise ValueError(f"attention exchange {exchange!r}")
    crowded = best["nq"] > CLUSTERS_RESIDENT.get(best["CL"], best["nq"])
    best["XM"] = "grid" if exchange == "grid" or (exchange == "auto" and fits and crowded) else "cluster"
    best["SMEM_LAUNCH"] = best["SMEM"]
    if best["XM"] == "grid":
        # CTAs of one tile wait on one another, and tcgen05.alloc waits for free columns: no SM
        # may hold more of these CTAs than its tensor memory serves, so pad the shared memory
        per_sm = TMEM_COLS_MAX // best["TCOLS"]
        best["SMEM_LAUNCH"] = max(best["SMEM"], SM_SMEM_BYTES // (per_sm + 1) - 1024 + 1)
    return best, why


_TC_HELPERS = r"""
#include <string.h>
#include "emmy_sm100.cuh"
namespace {
__device__ __forceinline__ void emmy_umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns: thread t of the warp gets lane (base + t)
__device__ __forceinline__ void emmy_tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ float4 emmy_ld4(const float *p, bool aligned) {
    return aligned ? *reinterpret_cast<const float4 *>(p) : make_float4(p[0], p[1], p[2], p[3]);
}
__device__ __forceinline__ void emmy_fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ float emmy_dsmem_ld(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr));
    return v;
}
// x = hi + lo exactly; hi keeps the 10 explicit mantissa bits a tf32 operand holds
__device__ __forceinline__ float emmy_tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }
// byte offset of word w (0..31) of row r in a 128-byte-swizzled K-major tile of 32-word rows
__device__ __forceinline__ uint32_t emmy_sw128(uint32_t r, uint32_t w) {
    return r * 128u + ((((w >> 2) ^ (r & 7u)) << 4) | ((w & 3u) << 2));
}
__device__ __forceinline__ void emmy_put_split(uint8_t *hi, uint8_t *lo, uint32_t off, float x) {
    const float h = emmy_tf32_hi(x);
    *reinterpret_cast<float *>(hi + off) = h;
    *reinterpret_cast<float *>(lo + off) = x - h;
}
__device__ __forceinline__ void emmy_put_split4(uint8_t *hi, uint8_t *lo, uint32_t off, float4 x) {
    const float4 h = make_float4(emmy_tf32_hi(x.x), emmy_tf32_hi(x.y), emmy_tf32_hi(x.z), emmy_tf32_hi(x.w));
    *reinterpret_cast<float4 *>(hi + off) = h;
    *reinterpret_cast<float4 *>(lo + off) = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
}
}  // namespace
"""

# barrier of the CTAs of one query tile under a cooperative launch (every CTA resident)
_GRID_HELPERS = r"""
namespace {
__device__ __forceinline__ unsigned emmy_ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Every thread of the CTA calls it.  *count only ever grows: every CTA of the tile adds 1 per
// barrier, so the n arrivals at one barrier return values in [i n, (i + 1) n) and the barrier is
// passed once the count reaches (i + 1) n (n a power of two: the wrap at 2^32 keeps this).  A
// launch leaves the count a multiple of n; one whose wait ran out may not, and the module must
// be loaded again before its next launch.  false: the wait ran out, now or in an earlier call
// of this launch (*failed is set then; later calls return at once).  The CTA's own
// tensor-core work does not depend on the other CTAs, so its mbarrier waits go on as usual.
__device__ __noinline__ bool emmy_group_sync(unsigned *count, unsigned n, volatile uint32_t *failed,
                                             uint64_t wait_ns) {
    __syncthreads();
    if (threadIdx.x == 0) {
        if (*failed == 0u) {
            __threadfence();
            const unsigned target = (atomicAdd(count, 1u) / n + 1u) * n;
            const uint64_t t0 = emmy::globaltimer();
            while ((int)(emmy_ld_acquire_gpu(count) - target) < 0) {
                if (emmy::globaltimer() - t0 > wait_ns) {
                    *failed = 1u;
                    break;
                }
                __nanosleep(32);
            }
            __threadfence();
        }
    }
    __syncthreads();
    return *failed == 0u;
}
}  // namespace
"""


# schedule knobs: every wait's limit, and a test-only switch under which CTA 1 leaves out its
# first arrival at its tile's barrier (grid exchange), so that the other CTAs' waits run out
TC_TUNE = {"wait_ns": 2_000_000_000, "skip_first_arrive": False}


def generate_tc(kop: ir.KernelOp, plan, lay: dict, shapes: dict, dtypes: dict, args: list[str],
                scalars: dict[str, str], written: set[str], tune: dict | None = None) -> KernelSource:
    from .attention import KeyLoop
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
    SQ, SK, D, DV = plan.SQ, plan.SK, plan.D, plan.DV
    CL, KC, DP, DVP = lay["CL"], lay["KC"], lay["DP"], lay["DVP"]
    grid_x = lay.get("XM", "cluster") == "grid"
    tune = {**TC_TUNE, **(tune or {})}
    if set(tune) - set(TC_TUNE):
        raise ValueError(f"unknown attention_tune keys: {sorted(set(tune) - set(TC_TUNE))}")
    if tune["skip_first_arrive"] and not grid_x:
        raise ValueError("skip_first_arrive needs the grid exchange")
    GMAX = lay["nq"] * CL
    NKB, NCH = DP // 32, KC // 32
    fus = fusable_products(kop.body)
    keyloops = [s for s in plan.steps if isinstance(s, KeyLoop)]
    last = keyloops[-1]
    wname = lay["W"]
    nacc = sum(len(st.row_accs) for st in keyloops)
    qp, kp, vp, op_ = ptrs[plan.q], ptrs[plan.kmat], ptrs[plan.v], ptrs[plan.out_name]
    L: list[str] = []
    w = L.append
    w(DEVICE_PRELUDE)
    w(_TC_HELPERS)
    w(f"""namespace {{
constexpr int SQ = {SQ}, SK = {SK}, D = {D}, DV = {DV}, DP = {DP}, DVP = {DVP};
constexpr int CL = {CL}, KC = {KC}, NKB = {NKB}, NCH = {NCH}, TCOLS = {lay['TCOLS']};
constexpr int T = {T}, NG = {NG}, NACC = {max(1, nacc)};
constexpr uint32_t R1 = {lay['R1']}u, R2 = {lay['R2']}u, NSTAT = {lay['NSTAT']}u, SMEM_BYTES = {lay['SMEM']}u;
constexpr uint32_t IDESC_S = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(KC >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t IDESC_O = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(DVP >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint64_t WAIT_NS = {int(tune["wait_ns"])}ull;
constexpr int UB = 4;   // float4 loads in flight per thread while operands are staged
constexpr int GMAX = {GMAX};  // CTAs of the whole problem (CL per query tile)
}}  // namespace
""")
    if grid_x:
        w(_GRID_HELPERS)
        w("""namespace {
// exchange through global memory: row values [CTA][NACC][128], partial outputs [CTA][DVP][128]
// (column-major, so a warp's stores are contiguous), and one arrival counter per tile
__device__ __align__(16) float emmy_attn_stats[GMAX * NACC * 128];
__device__ __align__(16) float emmy_attn_opart[(size_t)GMAX * DVP * 128];
__device__ unsigned int emmy_attn_sync[GMAX / CL];
}  // namespace
""")
    w(f'extern "C" __global__ void __launch_bounds__({T}, 1) ' + kop.name + "(" + ", ".join(sig) + ") {")
    w("    uint32_t dyn_smem;")
    w('    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));')
    w("    if (blockDim.x != T || blockDim.y != 1 || blockDim.z != 1 || dyn_smem < SMEM_BYTES ||")
    if grid_x:
        w("        gridDim.x > (unsigned)GMAX || gridDim.y != 1 || gridDim.z != 1 || (gridDim.x % CL) != 0) {")
    else:
        w("        emmy::cluster_nctarank() != (uint32_t)CL || (gridDim.x % CL) != 0) {")
    w("        if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) atomicOr(&emmy_status, EMMY_STATUS_BAD_LAUNCH);")
    w("        return;")
    w("    }")
    w("    const long long RB = (long long)(emmy_rb < (unsigned long long)SQ ? emmy_rb : SQ);")
    w("    const long long RE = (long long)(emmy_re < (unsigned long long)SQ ? emmy_re : SQ);")
    w("    extern __shared__ __align__(1024) uint8_t smem_raw[];")
    w("    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));")
    w("    uint8_t *const r1 = smem;            // Q hi/lo, then P hi/lo x 2, then the partial O")
    w("    uint8_t *const r2 = smem + R1;       // K hi/lo, then V hi/lo")
    w("    float *const stats = reinterpret_cast<float *>(smem + R1 + R2);      // [NACC][128]: cluster exchange")
    w("    float *const gpart = stats + NACC * 128;                             // [NACC][NG][128]: column groups")
    w("    // s_done, o_done, pfree0, pfree1 (MMA commits); pfull0, pfull1 (one arrival per warp)")
    w("    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem + R1 + R2 + NSTAT);")
    w("    uint32_t *const tmem_holder = reinterpret_cast<uint32_t *>(bars + 6);")
    w("    volatile uint32_t *const abort_flag = tmem_holder + 1;")
    if grid_x:
        w("    volatile uint32_t *const gfail = tmem_holder + 2;   // a wait for the tile's other CTAs ran out")
    w("    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;")
    w("    const int lq = warp & 3, grp = warp >> 2;        // tensor-memory lane quarter, key column group")
    w("    const int rloc = lq * 32 + lane;                 // this thread's query row in the tile")
    w(f"    const bool q_al = (reinterpret_cast<uintptr_t>({qp}) & 15u) == 0;   // 16-byte loads, else four 4-byte ones")
    w(f"    const bool k_al = (reinterpret_cast<uintptr_t>({kp}) & 15u) == 0;")
    w(f"    const bool v_al = (reinterpret_cast<uintptr_t>({vp}) & 15u) == 0;")
    w("    (void)q_al; (void)k_al; (void)v_al;")
    if grid_x:
        w("    const uint32_t crank = blockIdx.x % CL;           // this CTA's key chunk of its tile")
        w("    const uint32_t gbase = blockIdx.x - crank;        // first CTA of its tile")
        w("    unsigned *const gsync = emmy_attn_sync + blockIdx.x / CL;")
    else:
        w("    const uint32_t crank = emmy::cluster_ctarank();")
    w("    const int kbeg = (int)crank * KC;")
    w("    if (tid == 0) {")
    w("        for (int b = 0; b < 4; ++b) emmy::mbar_init(&bars[b], 1);")
    w("        for (int b = 4; b < 6; ++b) emmy::mbar_init(&bars[b], T / 32);")
    w("        *abort_flag = 0u;")
    if grid_x:
        w("        *gfail = 0u;")
    w("        emmy::fence_barrier_init();")
    w("    }")
    w("    if (warp == 0) { emmy::tmem_alloc(tmem_holder, TCOLS); emmy::tmem_relinquish(); }")
    w("    emmy::tc_fence_before();")
    w("    __syncthreads();")
    w("    emmy::tc_fence_after();")
    w("    const uint32_t tmem = *tmem_holder;")
    w("    const uint32_t trow = (uint32_t)(lq * 32) << 16;")
    w("    uint32_t ph_s = 0, ph_o = 0, pissued[2] = {0u, 0u}, pwaited[2] = {0u, 0u};")
    w("    bool ok = true;")
    if grid_x:
        w("    bool gok = true;   // every wait for the tile's other CTAs ended in time")
    w("    const int qt0 = (int)(RB / 128);")
    w("    const int nqt = RE > RB ? (int)((RE + 127) / 128) - qt0 : 0;")
    w("    for (int qt = qt0 + (int)(blockIdx.x / CL); qt < qt0 + nqt; qt += (int)(gridDim.x / CL)) {")
    w("        const long long q0 = (long long)qt * 128;")

    # each loop loads UB float4s per thread before it stores any, so a thread keeps UB loads
    # in flight (a loop that consumes each load at once waits out the memory latency per element)
    def batched(total: str, decode: list[str], load: list[str], store: list[str], ind: str = "        ") -> None:
        w(f"{ind}for (int e0 = tid; e0 < {total}; e0 += T * UB) {{")
        w(f"{ind}    float4 xb[UB];")
        w(f"{ind}    #pragma unroll")
        w(f"{ind}    for (int u = 0; u < UB; ++u) {{")
        w(f"{ind}        const int e = e0 + u * T;")
        w(f"{ind}        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);")
        w(f"{ind}        if (e < {total}) {{")
        for ln in decode + load:
            w(f"{ind}            {ln}")
        w(f"{ind}        }}")
        w(f"{ind}        xb[u] = x;")
        w(f"{ind}    }}")
        w(f"{ind}    #pragma unroll")
        w(f"{ind}    for (int u = 0; u < UB; ++u) {{")
        w(f"{ind}        const int e = e0 + u * T;")
        w(f"{ind}        if (e < {total}) {{")
        w(f"{ind}            const float4 x = xb[u];")
        for ln in decode + store:
            w(f"{ind}            {ln}")
        w(f"{ind}        }}")
        w(f"{ind}    }}")
        w(f"{ind}}}")

    def staged(tag: str, total: int, decode: list[str], load: list[str], ind: str = "        ") -> bool:
        """Loads of a whole operand into registers (at most 8 float4 per thread), stored later by
        ``staged_store``: the loads of several operands are then all in flight together."""
        n = -(-total // T)
        if n > 8:
            return False
        w(f"{ind}float4 {tag}[{n}];")
        w(f"{ind}#pragma unroll")
        w(f"{ind}for (int u = 0; u < {n}; ++u) {{")
        w(f"{ind}    const int e = tid + u * T;")
        w(f"{ind}    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);")
        w(f"{ind}    if (e < {total}) {{")
        for ln in decode + load:
            w(f"{ind}        {ln}")
        w(f"{ind}    }}")
        w(f"{ind}    {tag}[u] = x;")
        w(f"{ind}}}")
        return True

    def staged_store(tag: str, total: int, decode: list[str], store: list[str], ind: str = "        ") -> None:
        n = -(-total // T)
        w(f"{ind}#pragma unroll")
        w(f"{ind}for (int u = 0; u < {n}; ++u) {{")
        w(f"{ind}    const int e = tid + u * T;")
        w(f"{ind}    if (e < {total}) {{")
        w(f"{ind}        const float4 x = {tag}[u];")
        for ln in decode + store:
            w(f"{ind}        {ln}")
        w(f"{ind}    }}")
        w(f"{ind}}}")

    def operand(tag: str, total: int, decode, load, store, deferred: list) -> None:
        """Stage an operand in registers if it fits (its stores are emitted by ``flush``), else
        load and store it in batches right here."""
        if staged(tag, total, decode, load):
            deferred.append((tag, total, decode, store))
        else:
            batched(str(total), decode, load, store)

    def flush(deferred: list) -> None:
        for tag, total, decode, store in deferred:
            staged_store(tag, total, decode, store)
        deferred.clear()

    pending: list = []
    w("        // Q tile (A of S): 128 rows x DP, hi and lo; rows past SQ and columns past D are 0")
    operand("qreg", 128 * (DP // 4),
            ["const int r = e / (DP / 4), c4 = e % (DP / 4);", "const long long gr = q0 + r;"],
            [f"if (gr < SQ && 4 * c4 < D) x = emmy_ld4({qp} + gr * D + 4 * c4, q_al);"],
            ["const uint32_t off = (uint32_t)((4 * c4) / 32) * 16384u + emmy_sw128((uint32_t)r, (uint32_t)((4 * c4) % 32));",
             "emmy_put_split4(r1, r1 + NKB * 16384u, off, x);"], pending)
    w("        // this CTA's keys (B of S): KC rows (keys) x DP, hi and lo; keys past SK are 0")
    if plan.k_dk:
        # a warp takes 16 rows of kt (d) x 8 keys: two lanes read the 32 contiguous bytes of one
        # row (one sector per lane pair), and each lane stores its 4 keys as 4 words of 4 key
        # rows; the 32 stores of an instruction fall in 32 different banks (rows 4k and 4k + 4
        # differ in bit 2 of the swizzle)
        operand("kreg", DP * (KC // 4),
                ["const int grp_ = e >> 5, di = (e >> 1) & 15, kj = e & 1;",
                 "const int d = 16 * (grp_ % (DP / 16)) + di, k4 = 2 * (grp_ / (DP / 16)) + kj;",
                 "const int key0 = kbeg + 4 * k4;"],
                ["if (d < D) {",
                 "    if (key0 + 3 < SK) {",
                 f"        x = emmy_ld4({kp} + (long long)d * SK + key0, k_al && (SK % 4) == 0);",
                 "    } else {",
                 f"        if (key0 < SK) x.x = {kp}[(long long)d * SK + key0];",
                 f"        if (key0 + 1 < SK) x.y = {kp}[(long long)d * SK + key0 + 1];",
                 f"        if (key0 + 2 < SK) x.z = {kp}[(long long)d * SK + key0 + 2];",
                 "    }",
                 "}"],
                ["const float xs[4] = {x.x, x.y, x.z, x.w};",
                 "#pragma unroll",
                 "for (int q = 0; q < 4; ++q) {",
                 "    const uint32_t off = (uint32_t)(d / 32) * (KC * 128u) + emmy_sw128((uint32_t)(4 * k4 + q), (uint32_t)(d % 32));",
                 "    emmy_put_split(r2, r2 + NKB * KC * 128u, off, xs[q]);",
                 "}"], pending)
    else:
        operand("kreg", KC * (DP // 4),
                ["const int r = e / (DP / 4), c4 = e % (DP / 4);", "const int key = kbeg + r;"],
                [f"if (key < SK && 4 * c4 < D) x = emmy_ld4({kp} + (long long)key * D + 4 * c4, k_al);"],
                ["const uint32_t off = (uint32_t)((4 * c4) / 32) * (KC * 128u) + emmy_sw128((uint32_t)r, (uint32_t)((4 * c4) % 32));",
                 "emmy_put_split4(r2, r2 + NKB * KC * 128u, off, x);"], pending)
    flush(pending)
    w("        emmy_fence_async_smem();")
    w("        emmy::tc_fence_before();")
    w("        __syncthreads();")
    w("        if (tid == 0) {")
    w("            emmy::tc_fence_after();")
    w("            const uint32_t qh = emmy::smem_u32(r1), ql = qh + NKB * 16384u;")
    w("            const uint32_t kh = emmy::smem_u32(r2), kl = kh + NKB * KC * 128u;")
    w("            #pragma unroll 1")
    w("            for (int kb = 0; kb < NKB; ++kb) {")
    w("                #pragma unroll")
    w("                for (int kk = 0; kk < 4; ++kk) {")
    w("                    const uint32_t ao = kb * 16384u + kk * 32u, bo = kb * (KC * 128u) + kk * 32u;")
    w("                    const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;")
    w("                    emmy_umma_tf32(tmem, emmy::smem_desc_sw128(qh + ao, 16, 1024), emmy::smem_desc_sw128(kh + bo, 16, 1024), IDESC_S, acc);")
    w("                    emmy_umma_tf32(tmem, emmy::smem_desc_sw128(qh + ao, 16, 1024), emmy::smem_desc_sw128(kl + bo, 16, 1024), IDESC_S, 1u);")
    w("                    emmy_umma_tf32(tmem, emmy::smem_desc_sw128(ql + ao, 16, 1024), emmy::smem_desc_sw128(kh + bo, 16, 1024), IDESC_S, 1u);")
    w("                }")
    w("            }")
    w("            emmy::umma_commit(&bars[0]);")
    w("        }")
    w("        __syncwarp();")
    w("        // this CTA's v rows (B of O): DVP rows (columns of v) x KC keys in 32-key chunks, hi and lo;")
    w("        // consecutive threads take consecutive keys, so a warp's stores cover 32 words of the same rows.")
    w("        // Loaded while the score MMAs run, stored over the K operand once they are done")
    # a warp takes 16 keys x 8 columns of v: two lanes read 32 contiguous bytes of one key's row,
    # and each lane stores its 4 columns as one word of 4 operand rows (32 banks, as for K)
    v_decode = ["const int grp_ = e >> 5, ki = (e >> 1) & 15, jj = e & 1;",
                "const int kl_ = 16 * (grp_ % (KC / 16)) + ki, j4 = 2 * (grp_ / (KC / 16)) + jj;",
                "const int key = kbeg + kl_;"]
    v_load = [f"if (key < SK && 4 * j4 < DV) x = emmy_ld4({vp} + (long long)key * DV + 4 * j4, v_al);"]
    v_store = ["const float xs[4] = {x.x, x.y, x.z, x.w};",
               "#pragma unroll",
               "for (int q = 0; q < 4; ++q) {",
               "    const uint32_t off = (uint32_t)(kl_ / 32) * (DVP * 128u) + emmy_sw128((uint32_t)(4 * j4 + q), (uint32_t)(kl_ % 32));",
               "    emmy_put_split(r2, r2 + NCH * DVP * 128u, off, xs[q]);",
               "}"]
    v_early = staged("vreg", KC * (DVP // 4), v_decode, v_load)
    w("        if (!emmy::mbar_wait(&bars[0], ph_s, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) ok = false;")
    w("        ph_s ^= 1u;")
    w("        emmy::tc_fence_after();")
    if v_early:
        staged_store("vreg", KC * (DVP // 4), v_decode, v_store)
    else:
        batched(str(KC * (DVP // 4)), v_decode, v_load, v_store)
    w("        emmy_fence_async_smem();")
    w("        __syncthreads();")
    # ---- the IR's passes: thread (rloc, grp) takes keys [8 grp, 8 grp + 8) of every 32-key chunk
    w("        const long long row = q0 + rloc;")
    rem = Emitter(shapes, dtypes, ptrs, indent="        ")
    rem.fusable = fus
    rem.env.update(scalar_env)
    rem.bind_const(plan.i, "int", "row")
    slot = 0
    for st in plan.steps:
        if not isinstance(st, KeyLoop):
            s_ = st[1]
            if isinstance(s_, ir.Init) and s_.name in plan.cell_accs:
                continue
            rem.run((s_,))
            continue
        final = st is last
        accs = []
        L.extend(rem.lines)
        rem.lines = []
        for a, op in st.row_accs:
            accum = next(t for t in st.post if isinstance(t, ir.Accum) and t.name == a)
            accs.append((a, op, accum))
            w(f"        float part_{_c(a)} = {f32_lit(identity_of(op))};")
        w(f"        // key loop over {st.loop.axis.name}: scores from tensor memory, 8 keys of each 32-key chunk per thread")
        w("        #pragma unroll 1")
        w("        for (int ch = 0; ch < NCH; ++ch) {")
        w("            uint32_t sreg[8];")
        w("            emmy_tmem_ld_x8(tmem + trow + (uint32_t)(ch * 32 + 8 * grp), sreg);")
        w("            emmy::tmem_ld_wait();")
        if final:
            w("            float pw[8];")
        w("            #pragma unroll")
        w("            for (int kk = 0; kk < 8; ++kk) {")
        w("                const int key = kbeg + ch * 32 + 8 * grp + kk;")
        if final:
            w("                pw[kk] = 0.0f;")
        w("                if (key < SK) {")
        kem = Emitter(shapes, dtypes, ptrs, indent="                    ")
        kem.fusable = fus
        kem.env.update(rem.env)
        kem.declared = {}
        kem.bind_const(plan.i, "int", "row")
        kem.bind_const(st.loop.axis.name, "int", "(long long)key")
        kem.env[st.dot_acc] = ("f32", "__uint_as_float(sreg[kk])")
        kem.run(tuple(st.indep))
        L.extend(kem.lines)
        for a, op, accum in accs:
            prod = kem.plain_product(accum.value) if op == "add" else None
            if prod is not None:
                w(f"                    part_{_c(a)} = __fmaf_rn({prod[0]}, {prod[1]}, part_{_c(a)});")
            else:
                w(f"                    part_{_c(a)} = {combine_code(op, f'part_{_c(a)}', kem.as_f32(accum.value))};")
        if final:
            w(f"                    pw[kk] = {kem.as_f32(wname)};")
        w("                }")
        w("            }")
        if final:
            w("            // P chunk (A of O): words [8 grp, 8 grp + 8) of this row, hi and lo, into buffer ch & 1")
            w("            const int b = ch & 1;")
            w("            if (pissued[b] > pwaited[b]) {")
            w("                if (!emmy::mbar_wait(&bars[2 + b], pwaited[b] & 1u, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) ok = false;")
            w("                ++pwaited[b];")
            w("            }")
            w("            uint8_t *const ph = r1 + (uint32_t)b * 32768u, *const pl = ph + 16384u;")
            w("            emmy_put_split4(ph, pl, emmy_sw128((uint32_t)rloc, (uint32_t)(8 * grp)), make_float4(pw[0], pw[1], pw[2], pw[3]));")
            w("            emmy_put_split4(ph, pl, emmy_sw128((uint32_t)rloc, (uint32_t)(8 * grp + 4)), make_float4(pw[4], pw[5], pw[6], pw[7]));")
            w("            // each warp reports its part of the chunk; only the issuing thread waits for all")
            w("            emmy_fence_async_smem();")
            w("            emmy::tc_fence_before();")
            w("            __syncwarp();")
            w("            if (lane == 0) emmy::mbar_arrive(&bars[4 + b]);")
            w("            if (tid == 0) {")
            w("                if (!emmy::mbar_wait(&bars[4 + b], pissued[b] & 1u, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) ok = false;")
            w("                emmy::tc_fence_after();")
            w("                const uint32_t pa = emmy::smem_u32(ph), pb = emmy::smem_u32(pl);")
            w("                const uint32_t vh = emmy::smem_u32(r2) + (uint32_t)ch * (DVP * 128u);")
            w("                const uint32_t vl = vh + NCH * DVP * 128u;")
            w("                #pragma unroll")
            w("                for (int kk = 0; kk < 4; ++kk) {")
            w("                    const uint32_t acc = (ch | kk) != 0 ? 1u : 0u;")
            w("                    emmy_umma_tf32(tmem + KC, emmy::smem_desc_sw128(pa + kk * 32u, 16, 1024), emmy::smem_desc_sw128(vh + kk * 32u, 16, 1024), IDESC_O, acc);")
            w("                    emmy_umma_tf32(tmem + KC, emmy::smem_desc_sw128(pa + kk * 32u, 16, 1024), emmy::smem_desc_sw128(vl + kk * 32u, 16, 1024), IDESC_O, 1u);")
            w("                    emmy_umma_tf32(tmem + KC, emmy::smem_desc_sw128(pb + kk * 32u, 16, 1024), emmy::smem_desc_sw128(vh + kk * 32u, 16, 1024), IDESC_O, 1u);")
            w("                }")
            w("                emmy::umma_commit(&bars[2 + b]);")
            w("            }")
            w("            __syncwarp();")
            w("            ++pissued[b];")
        w("        }")
        if accs:
            w("        // row partials: the column groups in group order, then the cluster's CTAs in CTA order")
            for fi, (a, op, accum) in enumerate(accs):
                w(f"        gpart[({slot + fi} * NG + grp) * 128 + rloc] = part_{_c(a)};")
            w("        __syncthreads();")
            w("        if (grp == 0) {")
            for fi, (a, op, accum) in enumerate(accs):
                w(f"            float c = gpart[({slot + fi} * NG) * 128 + rloc];")
                w("            #pragma unroll")
                w("            for (int g = 1; g < NG; ++g)")
                w(f"                c = {combine_code(op, 'c', f'gpart[({slot + fi} * NG + g) * 128 + rloc]')};")
                if grid_x:
                    w(f"            emmy_attn_stats[((size_t)blockIdx.x * NACC + {slot + fi}) * 128 + rloc] = c;")
                else:
                    w(f"            stats[{slot + fi} * 128 + rloc] = c;")
            w("        }")
            if grid_x and tune["skip_first_arrive"] and slot == 0:
                w("        if (blockIdx.x == 1u && qt == qt0) __syncthreads();   // test build: no arrival")
                w("        else if (!emmy_group_sync(gsync, CL, gfail, WAIT_NS)) gok = false;")
            elif grid_x:
                w("        if (!emmy_group_sync(gsync, CL, gfail, WAIT_NS)) gok = false;")
            else:
                w("        emmy::cluster_sync();")
            for fi, (a, op, accum) in enumerate(accs):
                cur = rem.as_f32(a)
                w(f"        {{ float tot = {cur}, got[CL];")
                w("          #pragma unroll")
                if grid_x:
                    w(f"          for (int rr = 0; rr < CL; ++rr) got[rr] = __ldcg(&emmy_attn_stats[((size_t)(gbase + rr) * NACC + {slot + fi}) * 128 + rloc]);")
                else:
                    w(f"          for (int rr = 0; rr < CL; ++rr) got[rr] = emmy_dsmem_ld(emmy::mapa(&stats[{slot + fi} * 128 + rloc], (uint32_t)rr));")
                w("          #pragma unroll")
                w("          for (int rr = 0; rr < CL; ++rr)")
                w(f"              tot = {combine_code(op, 'tot', 'got[rr]')};")
                L.extend(rem.lines)
                rem.lines = []
                var = rem.declare(a, "f32")
                L.extend(rem.lines)
                rem.lines = []
                w(f"          {var} = tot; }}")
                rem.env[a] = ("f32", var)
            slot += len(accs)
    L.extend(rem.lines)
    rem.lines = []
    w("        // the partial O of this CTA's keys")
    w("        if (tid == 0) emmy::umma_commit(&bars[1]);")
    w("        __syncwarp();")
    w("        if (!emmy::mbar_wait(&bars[1], ph_o, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) ok = false;")
    w("        ph_o ^= 1u;")
    w("        for (int b = 0; b < 2; ++b)")
    w("            while (pwaited[b] < pissued[b]) {")
    w("                if (!emmy::mbar_wait(&bars[2 + b], pwaited[b] & 1u, abort_flag, EMMY_STATUS_TIMEOUT_MMA, WAIT_NS)) ok = false;")
    w("                ++pwaited[b];")
    w("            }")
    w("        emmy::tc_fence_after();")
    if grid_x:
        w("        float *const opart = emmy_attn_opart + (size_t)blockIdx.x * DVP * 128;")
    else:
        w("        float *const opart = reinterpret_cast<float *>(r1);")
    w("        if (grp * 32 < DVP) {")
    w("            uint32_t oreg[32];")
    w("            emmy::tmem_ld_32x32b_x32(tmem + trow + (uint32_t)(KC + 32 * grp), oreg);")
    w("            emmy::tmem_ld_wait();")
    w("            #pragma unroll")
    w("            for (int jj = 0; jj < 32; ++jj)")
    if grid_x:
        w("                if (32 * grp + jj < DVP) opart[(32 * grp + jj) * 128 + rloc] = __uint_as_float(oreg[jj]);")
    else:
        w("                if (32 * grp + jj < DVP) opart[rloc * DVP + 32 * grp + jj] = __uint_as_float(oreg[jj]);")
    w("        }")
    if DVP > 32 * NG:
        raise UnsupportedIR(f"head size {DV} above {32 * NG}")
    w("        emmy::tc_fence_before();")
    if grid_x:
        w("        if (!emmy_group_sync(gsync, CL, gfail, WAIT_NS)) gok = false;")
    else:
        w("        emmy::cluster_sync();")
    w("        // rows [crank * 128 / CL, (crank + 1) * 128 / CL): the CL partials added in CTA order")
    w("        for (int e = tid; e < (128 / CL) * DV; e += T) {")
    if grid_x:
        w("            const int r = (int)crank * (128 / CL) + e % (128 / CL), jj = e / (128 / CL);")
    else:
        w("            const int r = (int)crank * (128 / CL) + e / DV, jj = e % DV;")
    w("            float tot = 0.0f, got[CL];")
    w("            #pragma unroll")
    if grid_x:
        w("            for (int rr = 0; rr < CL; ++rr) got[rr] = __ldcg(&emmy_attn_opart[(size_t)(gbase + rr) * DVP * 128 + jj * 128 + r]);")
    else:
        w("            for (int rr = 0; rr < CL; ++rr) got[rr] = emmy_dsmem_ld(emmy::mapa(&opart[r * DVP + jj], (uint32_t)rr));")
    w("            #pragma unroll")
    w("            for (int rr = 0; rr < CL; ++rr) tot += got[rr];")
    w(f"            if (q0 + r < RE && q0 + r >= RB) {op_}[(q0 + r) * DV + jj] = tot;")
    w("        }")
    if grid_x:
        w("        // the next tile reuses the exchange slots: wait until every CTA of this one has read them")
        w("        if (qt + (int)(gridDim.x / CL) < qt0 + nqt) {")
        w("            if (!emmy_group_sync(gsync, CL, gfail, WAIT_NS)) gok = false;")
        w("        }")
    else:
        w("        emmy::cluster_sync();")
    w("    }")
    w("    if (!ok) atomicOr(&emmy_status, EMMY_STATUS_TIMEOUT_MMA);")
    if grid_x:
        w("    if (!gok) atomicOr(&emmy_status, EMMY_STATUS_TIMEOUT_REDUCE);")
    w("    emmy::tc_fence_before();")
    w("    __syncthreads();")
    w("    if (warp == 0) { emmy::tc_fence_after(); emmy::tmem_dealloc(tmem, TCOLS); }")
    w("}")
    grid = lay["nq"] * CL
    rb = []
    for name in args:
        if name == plan.q:
            rb.append(D * 4)
        elif name == plan.out_name:
            rb.append(DV * 4)
        else:
            rb.append(0)
    launch = LaunchPlan(grid=(grid, 1, 1), block=(T, 1, 1), smem=lay.get("SMEM_LAUNCH", lay["SMEM"]),
                        cluster=(1, 1, 1) if grid_x else (CL, 1, 1), cooperative=grid_x,
                        range_total=SQ, range_align=128, range_bytes=rb)
    L.append(launch_record_source("attention", launch, params))
    notes = {"kernel": "attention_tcgen05_tf32x3", "cluster": 1 if grid_x else CL,
             "exchange": "grid" if grid_x else "cluster",
             "ctas_per_tile": CL, "keys_per_cta": KC, "query_tile": 128, "tune": tune,
             "threads": T, "smem": lay["SMEM"], "tmem_cols": lay["TCOLS"], "weights": wname}
    return KernelSource(entry=kop.name, source="\n".join(L), launch=launch, params=params,
                        family="attention", notes=notes)
