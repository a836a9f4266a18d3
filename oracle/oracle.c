/*
 * CPU restatement of the arithmetic in the reference compiler's emitted PTX.
 *
 * TEST INFRASTRUCTURE ONLY - the checker for tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference arm.  The product never links or
 * calls this code.
 *
 * Every function follows one piece of vedantgpt/emmy-ptx-compiler's
 * compile.py (line numbers cited per function).  The reference emits f32
 * instructions with round-to-nearest semantics; C float arithmetic with
 * FLT_EVAL_METHOD 0 (x86-64 SSE) and fmaf() give the same roundings, so the
 * integer-exact parts (add/sub/mul/div/sqrt/max/min, fma sequences, the
 * reduction order) reproduce the GPU results bit for bit.  The approximate
 * PTX instructions (ex2.approx.ftz, lg2.approx.ftz, rsqrt.approx.ftz) have
 * no published bit-exact definition, so they are restated with the
 * correctly-rounded libm functions plus flush-to-zero; callers compare
 * those results with an ulp tolerance.
 *
 * Build: make -C oracle   (gcc, no other dependencies)
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static float ftz(float x) {
    return (fpclassify(x) == FP_SUBNORMAL) ? copysignf(0.0f, x) : x;
}

/* fma.rn.f32 (compile.py:1280, 1300). */
void ora_fma_f32(const float *a, const float *b, const float *c, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fmaf(a[i], b[i], c[i]);
}

/* ex2.approx.ftz.f32 (compile.py:2099, 2104, 2151, 2165, 2177, 2195). */
void ora_ex2_f32(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ftz(exp2f(ftz(x[i])));
}

/* lg2.approx.ftz.f32 (compile.py:2138, 2141, 2192). */
void ora_lg2_f32(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ftz(log2f(ftz(x[i])));
}

/* rsqrt.approx.ftz.f32 (compile.py:2108). */
void ora_rsqrt_f32(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ftz((float)(1.0 / sqrt((double)ftz(x[i]))));
}

/* The naive-matmul schedule: one output per thread, acc = 0 (Init,
 * compile.py:1935-1940), then for kk = 0..K-1 in order
 * acc = fma.rn(A[i,kk], B[kk,j], acc)  (Loop + Load + multiply/Accum
 * contraction, compile.py:1813-1864, 1263-1283).  b_nk != 0 means B is
 * stored [N, K]. */
void ora_gemm_seqfma_f32(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K,
                         int b_nk) {
    for (int64_t i = 0; i < M; ++i) {
        const float *a = A + i * K;
        for (int64_t j = 0; j < N; ++j) {
            float acc = 0.0f;
            if (b_nk) {
                const float *b = B + j * K;
                for (int64_t k = 0; k < K; ++k) acc = fmaf(a[k], b[k], acc);
            } else {
                for (int64_t k = 0; k < K; ++k) acc = fmaf(a[k], B[k * N + j], acc);
            }
            C[i * N + j] = acc;
        }
    }
}

static float combine(int op, float a, float b) {
    switch (op) {
        case 4: return a + b;        /* fma-accumulated sums combine with add */
        case 1: return fmaxf(a, b);  /* max.f32 */
        case 2: return fminf(a, b);  /* min.f32 */
        case 3: return a * b;        /* mul.f32 */
        default: return a + b;       /* add.f32 */
    }
}

/* The cooperative strided reduction schedule with block_threads = bt and
 * warps of 32 (compile.py:1866-1914 StridedLoop, 2201-2211 Accum,
 * 2213-2230 WarpShuffle, 2232-2277 TreeHalve):
 *   thread t: acc = identity; for k = t; k < cols; k += bt: acc = acc (op) x[k]
 *   butterfly in each warp: for s = 16,8,4,2,1: acc = acc (op) shfl_xor(acc, s)
 *   warp leaders store to smem[w]; tree: for s = nw/2..1: smem[w] = smem[w] (op) smem[w+s]
 * out[row] = smem[0].  op: 0 add, 1 max, 2 min, 3 mul; 4 = the multiply/Accum
 * contraction acc = fma(x, y, acc) per element (compile.py:1263-1283),
 * combined with add across threads. */
void ora_strided_reduce_f32(const float *x, const float *y, int64_t rows, int64_t cols, int bt, int op,
                            float ident, float *out) {
    const int nw = bt / 32;
    for (int64_t r = 0; r < rows; ++r) {
        float acc[1024];
        float smem[32];
        const float *row = x + r * cols;
        for (int t = 0; t < bt; ++t) {
            float a = ident;
            if (op == 4) {
                const float *yr = y + r * cols;
                for (int64_t k = t; k < cols; k += bt) a = fmaf(row[k], yr[k], a);
            } else {
                for (int64_t k = t; k < cols; k += bt) a = combine(op, a, row[k]);
            }
            acc[t] = a;
        }
        for (int s = 16; s > 0; s >>= 1) {
            float nxt[1024];
            for (int t = 0; t < bt; ++t) nxt[t] = combine(op, acc[t], acc[(t & ~31) | ((t & 31) ^ s)]);
            memcpy(acc, nxt, sizeof(float) * (size_t)bt);
        }
        for (int w = 0; w < nw; ++w) smem[w] = acc[w * 32];
        for (int s = nw / 2; s > 0; s >>= 1)
            for (int w = 0; w < s; ++w) smem[w] = combine(op, smem[w], smem[w + s]);
        out[r] = smem[0];
    }
}

/* Sequential f32 accumulation of one row per thread (Loop schedule,
 * compile.py:1813-1864 with Accum 2201-2211); op 4 accumulates
 * fma(x, y, acc), the multiply/Accum contraction (1263-1283). */
void ora_loop_reduce_f32(const float *x, const float *y, int64_t rows, int64_t cols, int op, float seed,
                         float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        float acc = seed;
        const float *row = x + r * cols;
        const float *yr = y ? y + r * cols : 0;
        for (int64_t k = 0; k < cols; ++k)
            acc = (op == 4) ? fmaf(row[k], yr[k], acc) : combine(op, acc, row[k]);
        out[r] = acc;
    }
}

/* f64 row sums: the exact-ish reference the fixtures' expected values use
 * (tools/make_proxy_set.py:256, 335). */
void ora_row_sum_f64(const float *x, int64_t rows, int64_t cols, double *out) {
    for (int64_t r = 0; r < rows; ++r) {
        double s = 0.0;
        const float *row = x + r * cols;
        for (int64_t k = 0; k < cols; ++k) s += (double)row[k];
        out[r] = s;
    }
}

/* The naive attention IR (tools/make_proxy_set.py:416-474) as the reference
 * lowers it: every Loop runs in order (compile.py:1813-1864), multiply +
 * Accum pairs contract to fma.rn (compile.py:1263-1283), exp is ex2.approx of
 * x * log2(e) (compile.py:2099-2104), reciprocal is rcp.rn (compile.py:2106).
 * For output cell (i, j) the reference recomputes, in each of three passes
 * over the keys, s = (fma chain over d of q[i, d] * kt[d, k]) * scale:
 *   pass 1: m = max(m, s), m seeded -1e30 (compile.py:332);
 *   pass 2: den = den + exp(s - m), den seeded 0;
 *   then invd = 1 / den;
 *   pass 3: acc = fma(exp(s - m) * invd, v[k, j], acc), acc seeded 0.
 * s and exp(s - m) do not depend on j, so they are computed once per (i, k)
 * here; the values are the same.  kt is [d, sk] (the IR's layout); v is
 * [sk, dv].  Returns 0, or -1 when scratch memory is not available. */
int ora_attn_naive_f32(const float *q, const float *kt, const float *v, float *out, int64_t sq, int64_t sk,
                       int64_t d, int64_t dv, float scale) {
    const float L2E = 1.44269502162933349609375f; /* 0x3FB8AA3B: log2(e) rounded to f32 */
    float *s = (float *)malloc((size_t)sk * 2 * sizeof(float));
    if (!s) return -1;
    float *ex = s + sk;
    for (int64_t i = 0; i < sq; ++i) {
        float m = -1e30f;
        for (int64_t k = 0; k < sk; ++k) {
            float acc = 0.0f;
            for (int64_t t = 0; t < d; ++t) acc = fmaf(q[i * d + t], kt[t * sk + k], acc);
            s[k] = acc * scale;
            m = fmaxf(m, s[k]);
        }
        float den = 0.0f;
        for (int64_t k = 0; k < sk; ++k) {
            const float dl = s[k] - m;
            ex[k] = ftz(exp2f(ftz(dl * L2E)));
            den = den + ex[k];
        }
        const float invd = 1.0f / den;
        for (int64_t j = 0; j < dv; ++j) {
            float acc = 0.0f;
            for (int64_t k = 0; k < sk; ++k) acc = fmaf(ex[k] * invd, v[k * dv + j], acc);
            out[i * dv + j] = acc;
        }
    }
    free(s);
    return 0;
}

int ora_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
