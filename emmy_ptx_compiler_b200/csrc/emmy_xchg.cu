// Full-array f32 sum fused with its cross-GPU combine over NVLink peer memory,
// and the exchange group that compiled modules use for the same combine.
//
// The C4 step on N GPUs is: every GPU sums its shard, then the N partial sums
// are added so that every GPU holds the total.  emmy_sum_f32_allreduce does
// both in ONE kernel per GPU:
//
//   1. CTAs sum fixed-size chunks of the shard (four 128-bit streaming loads
//      in flight per thread, lane butterflies) and store per-chunk partials;
//      the CTA that finishes the last chunk adds the partials in chunk order
//      (the reduction family's last-block combine scheme);
//   2. that CTA's thread 0 exchanges the GPU's total with every other GPU
//      through their exchange buffers (emmy_xchg_dev.cuh: one 64-bit
//      epoch+value store per peer, a bounded wait for every peer's word) and
//      adds the N totals in rank order, so all GPUs get the same bits.
//
// emmy_launch_xchg (emmy_runtime.cpp) runs the same exchange at the end of a
// compiled full-array reduction KernelOp (its <entry>__xchg kernel); this
// file owns the exchange buffers and hands their addresses over through
// emmy_xchg_fill_args.
//
// A wait that runs out marks the GPU's group as failed (no more publishing
// until emmy_xchg_reset), sets bit 0 of the status word and writes NaN to the
// outputs; the kernel then returns, so the context stays usable.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "emmy_b200.h"
#include "emmy_xchg_dev.cuh"

extern "C" int emmy_record_error(int code, const char *msg);  // emmy_runtime.cpp (not exported)

namespace {

constexpr int kMaxRanks = EMMY_XCHG_MAX_RANKS;
constexpr int kMaxChunks = 4096;
constexpr uint64_t kMinChunk = 1ull << 14;
constexpr int kThreads = 256;
constexpr int kSms = 148;
constexpr int kBlocksPerSm = 8;
constexpr size_t kXchgBytes = EMMY_XCHG_BUFFER_BYTES;
static_assert(EMMY_XCHG_MAX_RANKS_DEV == EMMY_XCHG_MAX_RANKS, "exchange rank limit");
// scratch layout (bytes)
constexpr size_t kCounterOff = (kMaxChunks * sizeof(float) + 255) / 256 * 256;
constexpr size_t kScratchBytes = kCounterOff + 256;

struct Peers {
    unsigned char *buf[kMaxRanks];
};

int report(int code, const char *fmt, ...) {
    char msg[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    return emmy_record_error(code, msg);
}

__device__ __forceinline__ float warp_sum(float v) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

__device__ float block_sum(float v, float *s_warp) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) s_warp[wid] = v;
    __syncthreads();
    float r = 0.0f;
    if (wid == 0) {
        r = lane < nw ? s_warp[lane] : 0.0f;
        r = warp_sum(r);
    }
    return r;
}

__global__ void __launch_bounds__(kThreads) sum_allreduce_kernel(
    const float *__restrict__ x, uint64_t n, uint64_t chunk, uint32_t nchunks, float *__restrict__ out,
    unsigned char *scratch, EmmyXchgArgs xa) {
    __shared__ float s_warp[32];
    __shared__ int s_last;
    float *partials = reinterpret_cast<float *>(scratch);
    unsigned int *arrivals = reinterpret_cast<unsigned int *>(scratch + kCounterOff);
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) && (chunk % 4 == 0);
    for (uint32_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t k0 = static_cast<uint64_t>(c) * chunk;
        const uint64_t k1 = (k0 + chunk < n) ? (k0 + chunk) : n;
        float a[4][4] = {};
        uint64_t k;
        if (vec) {
            const uint64_t kv_end = k0 + (k1 - k0) / 4 * 4;
            const uint64_t step = 4ull * blockDim.x;
            k = k0 + 4ull * threadIdx.x;
            // four 16-byte loads in flight per thread
            for (; k + 3 * step + 3 < kv_end; k += 4 * step) {
                float4 v[4];
                #pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = __ldcs(reinterpret_cast<const float4 *>(x + k + u * step));
                #pragma unroll
                for (int u = 0; u < 4; ++u) {
                    a[u][0] += v[u].x;
                    a[u][1] += v[u].y;
                    a[u][2] += v[u].z;
                    a[u][3] += v[u].w;
                }
            }
            for (; k + 3 < kv_end; k += step) {
                const float4 v = __ldcs(reinterpret_cast<const float4 *>(x + k));
                a[0][0] += v.x;
                a[0][1] += v.y;
                a[0][2] += v.z;
                a[0][3] += v.w;
            }
            for (k = kv_end + threadIdx.x; k < k1; k += blockDim.x) a[0][0] += x[k];
        } else {
            for (k = k0 + threadIdx.x; k < k1; k += blockDim.x) a[0][0] += __ldcs(x + k);
        }
        float t = 0.0f;
        #pragma unroll
        for (int u = 0; u < 4; ++u) t += (a[u][0] + a[u][1]) + (a[u][2] + a[u][3]);
        const float total = block_sum(t, s_warp);
        if (threadIdx.x == 0) {
            __stcg(&partials[c], total);
            __threadfence();
            const unsigned prev = atomicAdd(arrivals, 1u);
            s_last = (prev == nchunks - 1);
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            float f = 0.0f;
            for (uint32_t i = threadIdx.x; i < nchunks; i += blockDim.x) f += __ldcg(&partials[i]);
            f = block_sum(f, s_warp);
            if (threadIdx.x == 0) {
                *arrivals = 0u;
                float got[EMMY_XCHG_MAX_RANKS_DEV];
                if (emmy_xchg_exchange(xa, &f, 1, got)) {
                    float s = got[0];
                    for (uint32_t r = 1; r < xa.nranks; ++r) s = __fadd_rn(s, got[r]);
                    *out = s;
                } else {
                    *out = __int_as_float(0x7fffffff);
                }
            }
        }
        __syncthreads();
    }
}

}  // namespace

struct emmy_xchg {
    int dev = 0, nranks = 1, rank = 0;
    unsigned char *local = nullptr;    // this GPU's exchange buffer (IPC-exported)
    unsigned char *scratch = nullptr;  // per-chunk partials + arrival counter
    Peers peers{};
    bool opened[kMaxRanks] = {false};
    bool connected = false;
    uint32_t epoch = 0;
    cudaIpcMemHandle_t handle{};
};

namespace {

struct DeviceGuard {
    int prev = 0;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
    }
    ~DeviceGuard() {
        if (ok) cudaSetDevice(prev);
    }
};

// Parameters of the next call: the group's buffers and a fresh epoch (0 is the
// value of a word nobody wrote, so it is skipped).
void next_args(emmy_xchg *x, int timeout_ms, EmmyXchgArgs *xa) {
    std::memset(xa, 0, sizeof *xa);
    for (int r = 0; r < x->nranks; ++r) xa->peer[r] = reinterpret_cast<unsigned long long>(x->peers.buf[r]);
    xa->local = reinterpret_cast<unsigned long long>(x->local);
    xa->rank = static_cast<unsigned>(x->rank);
    xa->nranks = static_cast<unsigned>(x->nranks);
    x->epoch += 1u;
    if (x->epoch == 0u) x->epoch = 1u;
    xa->epoch = x->epoch;
    xa->timeout_ns = static_cast<unsigned long long>(timeout_ms) * 1000000ull;
}

}  // namespace

extern "C" int emmy_xchg_create(int dev, int nranks, int rank, emmy_xchg_t *out, uint8_t handle[EMMY_XCHG_HANDLE_BYTES]) {
    if (!out || !handle) return report(EMMY_ERR_INVALID, "emmy_xchg_create: NULL argument");
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return report(EMMY_ERR_INVALID, "emmy_xchg_create: rank %d of %d (at most %d ranks)", rank, nranks, kMaxRanks);
    static_assert(sizeof(cudaIpcMemHandle_t) == EMMY_XCHG_HANDLE_BYTES, "IPC handle size");
    DeviceGuard g(dev);
    if (!g.ok) return report(EMMY_ERR_CUDA, "emmy_xchg_create: cannot make device %d current", dev);
    emmy_xchg *x = new emmy_xchg;
    x->dev = dev;
    x->nranks = nranks;
    x->rank = rank;
    cudaError_t e = cudaMalloc(&x->local, kXchgBytes);
    if (e == cudaSuccess) e = cudaMemset(x->local, 0, kXchgBytes);
    if (e == cudaSuccess) e = cudaMalloc(&x->scratch, kScratchBytes);
    if (e == cudaSuccess) e = cudaMemset(x->scratch, 0, kScratchBytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&x->handle, x->local);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (x->local) cudaFree(x->local);
        if (x->scratch) cudaFree(x->scratch);
        delete x;
        return report(EMMY_ERR_CUDA, "emmy_xchg_create: %s", cudaGetErrorString(e));
    }
    std::memcpy(handle, &x->handle, EMMY_XCHG_HANDLE_BYTES);
    *out = x;
    return EMMY_OK;
}

extern "C" int emmy_xchg_connect(emmy_xchg_t x, const uint8_t *handles) {
    if (!x || !handles) return report(EMMY_ERR_INVALID, "emmy_xchg_connect: NULL argument");
    DeviceGuard g(x->dev);
    if (!g.ok) return report(EMMY_ERR_CUDA, "emmy_xchg_connect: cannot make device %d current", x->dev);
    for (int r = 0; r < x->nranks; ++r) {
        const uint8_t *h = handles + static_cast<size_t>(r) * EMMY_XCHG_HANDLE_BYTES;
        if (r == x->rank || std::memcmp(h, &x->handle, EMMY_XCHG_HANDLE_BYTES) == 0) {
            // this GPU's own buffer (a handle equal to ours names it too)
            x->peers.buf[r] = x->local;
            continue;
        }
        cudaIpcMemHandle_t ih;
        std::memcpy(&ih, h, sizeof ih);
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return report(EMMY_ERR_CUDA, "emmy_xchg_connect: opening rank %d's buffer: %s", r, cudaGetErrorString(e));
        x->peers.buf[r] = static_cast<unsigned char *>(p);
        x->opened[r] = true;
    }
    x->connected = true;
    return EMMY_OK;
}

extern "C" int emmy_sum_f32_allreduce(emmy_xchg_t x, const float *data, uint64_t n, float *out, int timeout_ms,
                                      uint64_t stream) {
    if (!x || !out || (n > 0 && !data)) return report(EMMY_ERR_INVALID, "emmy_sum_f32_allreduce: NULL argument");
    if (!x->connected) return report(EMMY_ERR_INVALID, "emmy_sum_f32_allreduce: emmy_xchg_connect first");
    if (timeout_ms <= 0) timeout_ms = 1000;
    DeviceGuard g(x->dev);
    if (!g.ok) return report(EMMY_ERR_CUDA, "emmy_sum_f32_allreduce: cannot make device %d current", x->dev);
    uint64_t target = static_cast<uint64_t>(kSms) * kBlocksPerSm;
    uint64_t chunk = (n + target - 1) / (target ? target : 1);
    if (chunk < kMinChunk) chunk = kMinChunk;
    chunk = (chunk + 3) / 4 * 4;
    uint64_t nchunks = n ? (n + chunk - 1) / chunk : 1;
    if (nchunks > kMaxChunks) {
        chunk = (n + kMaxChunks - 1) / kMaxChunks;
        chunk = (chunk + 3) / 4 * 4;
        nchunks = (n + chunk - 1) / chunk;
    }
    const unsigned grid = static_cast<unsigned>(nchunks < target ? nchunks : target);
    EmmyXchgArgs xa;
    next_args(x, timeout_ms, &xa);
    sum_allreduce_kernel<<<grid, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        data, n, chunk, static_cast<uint32_t>(nchunks), out, x->scratch, xa);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return report(EMMY_ERR_CUDA, "emmy_sum_f32_allreduce launch: %s", cudaGetErrorString(e));
    return EMMY_OK;
}

// The next call's kernel parameter for a compiled module's <entry>__xchg kernel
// (emmy_launch_xchg in emmy_runtime.cpp).  Not exported.
extern "C" __attribute__((visibility("hidden"))) int emmy_xchg_fill_args(emmy_xchg_t x, int dev, int timeout_ms,
                                                                          void *args, size_t bytes) {
    if (!x || !args || bytes != sizeof(EmmyXchgArgs)) return report(EMMY_ERR_INVALID, "emmy_launch_xchg: bad exchange");
    if (!x->connected) return report(EMMY_ERR_INVALID, "emmy_launch_xchg: emmy_xchg_connect first");
    if (x->dev != dev)
        return report(EMMY_ERR_INVALID, "emmy_launch_xchg: exchange is on device %d, module on %d", x->dev, dev);
    next_args(x, timeout_ms <= 0 ? 1000 : timeout_ms, static_cast<EmmyXchgArgs *>(args));
    return EMMY_OK;
}

extern "C" int emmy_xchg_reset(emmy_xchg_t x) {
    if (!x) return report(EMMY_ERR_INVALID, "emmy_xchg_reset: NULL argument");
    DeviceGuard g(x->dev);
    if (!g.ok) return report(EMMY_ERR_CUDA, "emmy_xchg_reset: cannot make device %d current", x->dev);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemset(x->local, 0, kXchgBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return report(EMMY_ERR_CUDA, "emmy_xchg_reset: %s", cudaGetErrorString(e));
    x->epoch = 0;
    return EMMY_OK;
}

extern "C" int emmy_xchg_status(emmy_xchg_t x, uint32_t *status) {
    if (!x || !status) return report(EMMY_ERR_INVALID, "emmy_xchg_status: NULL argument");
    DeviceGuard g(x->dev);
    if (!g.ok) return report(EMMY_ERR_CUDA, "emmy_xchg_status: cannot make device %d current", x->dev);
    uint32_t v = 0, zero = 0;
    cudaError_t e = cudaMemcpy(&v, x->local + EMMY_XCHG_STATUS_OFF, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(x->local + EMMY_XCHG_STATUS_OFF, &zero, 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return report(EMMY_ERR_CUDA, "emmy_xchg_status: %s", cudaGetErrorString(e));
    *status = v;
    return EMMY_OK;
}

extern "C" int emmy_xchg_destroy(emmy_xchg_t x) {
    if (!x) return EMMY_OK;
    DeviceGuard g(x->dev);
    cudaDeviceSynchronize();
    for (int r = 0; r < kMaxRanks; ++r)
        if (x->opened[r]) cudaIpcCloseMemHandle(x->peers.buf[r]);
    if (x->local) cudaFree(x->local);
    if (x->scratch) cudaFree(x->scratch);
    delete x;
    return EMMY_OK;
}
