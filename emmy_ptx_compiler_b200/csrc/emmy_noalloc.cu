// emmy_sum_f32_noalloc: the full-array f32 sum of the reduction family for
// callers that cannot allocate device memory.
//
// Who needs it: hosts that embed this library but may not call cudaMalloc
// or any allocating routine - a caller running under a fixed memory budget
// with a pre-sized pool, a real-time loop where an allocation could block
// or fragment, or a runtime that owns every device allocation itself and
// hands out only input and output buffers.  The module-based path
// (emmy_load + emmy_launch) keeps its cross-block partials in globals of the
// loaded module; this entry point instead keeps them in a fixed array that
// is part of libemmy_b200 itself, so nothing is allocated per call.
//
// Scratch: one file-scope __device__ array of EMMY_NOALLOC_SCRATCH_BYTES
// (16 KiB of per-chunk partials + one 256-byte-aligned arrival counter).
// Every GPU that loads the library holds that array until the process exits.
// It is shared by every call on a device and keeps the last call's
// contents; the arrival counter is cleared at the start of each call.
// Calls that overlap on the GPU (different streams, or different host
// threads, on the same device) race on it and must be serialised by the
// caller.
//
// Limit: n may be at most EMMY_NOALLOC_MAX_ELEMENTS (2^36 floats, more than
// one GPU holds); larger sizes are rejected with EMMY_ERR_INVALID before
// anything is launched.  At most 1184 of the 4096 partial slots are used.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress (with that device current) and caches it; do
// that first call before any stream capture.  The cached address belongs to
// the device's primary context as it was then: after cudaDeviceReset (or any
// other reset of that context) the entry point must not be called again on
// that device in this process.  No call allocates: no
// cudaMalloc, cudaFree or allocating library routine is used.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "emmy_b200.h"

extern "C" int emmy_record_error(int code, const char *msg);  // emmy_runtime.cpp (not exported)

namespace {

constexpr int kMaxChunks = EMMY_NOALLOC_MAX_CHUNKS;  // partial slots in the scratch
constexpr uint64_t kMinChunk = 1ull << 14;           // elements per chunk, at least
constexpr int kThreads = 256;
constexpr int kBlocksPerSm = 8;
constexpr int kSms = 148;
constexpr size_t kCounterOffset = (kMaxChunks * sizeof(float) + 255) / 256 * 256;
static_assert(kCounterOffset + 256 <= EMMY_NOALLOC_SCRATCH_BYTES, "scratch layout");

// The scratch array.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[EMMY_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void *g_scratch_ptr[64] = {nullptr};

int report(int code, const char *fmt, ...);

__device__ __forceinline__ float warp_sum(float v) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Block-wide sum in a fixed order (lane butterflies, then warp 0 over the
// per-warp values); valid in thread 0.
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

// One CTA per chunk at a time (grid-stride over chunks).  Chunk c sums
// x[c*chunk, min(n, (c+1)*chunk)) in a fixed thread/order layout, writes its
// partial, and the CTA that completes the last chunk adds the partials in
// chunk order and stores the total.
__global__ void __launch_bounds__(kThreads) noalloc_sum_kernel(const float *__restrict__ x, uint64_t n,
                                                               uint64_t chunk, uint32_t nchunks,
                                                               float *__restrict__ out,
                                                               unsigned char *scratch) {
    __shared__ float s_warp[32];
    __shared__ int s_last;
    float *partials = reinterpret_cast<float *>(scratch);
    unsigned int *arrivals = reinterpret_cast<unsigned int *>(scratch + kCounterOffset);
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) && (chunk % 4 == 0);
    for (uint32_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t k0 = static_cast<uint64_t>(c) * chunk;
        const uint64_t k1 = (k0 + chunk < n) ? (k0 + chunk) : n;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        uint64_t k = k0;
        if (vec) {
            const uint64_t kv_end = k0 + (k1 - k0) / 4 * 4;
            for (k = k0 + 4ull * threadIdx.x; k + 3 < kv_end; k += 4ull * blockDim.x) {
                const float4 v = __ldcs(reinterpret_cast<const float4 *>(x + k));
                a0 += v.x;
                a1 += v.y;
                a2 += v.z;
                a3 += v.w;
            }
            for (k = kv_end + threadIdx.x; k < k1; k += blockDim.x) a0 += x[k];
        } else {
            for (k = k0 + threadIdx.x; k < k1; k += blockDim.x) a0 += __ldcs(x + k);
        }
        const float total = block_sum((a0 + a1) + (a2 + a3), s_warp);
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
                *out = f;
                *arrivals = 0u;
            }
        }
        __syncthreads();
    }
}

}  // namespace

extern "C" int emmy_sum_f32_noalloc(int dev, const float *x, uint64_t n, float *out, uint64_t stream) {
    if (!out || (n > 0 && !x)) return report(EMMY_ERR_INVALID, "emmy_sum_f32_noalloc: NULL pointer");
    if (n > EMMY_NOALLOC_MAX_ELEMENTS)
        return report(EMMY_ERR_INVALID,
                      "emmy_sum_f32_noalloc: n = %llu exceeds the maximum of %llu elements this entry point "
                      "supports with its fixed %d-byte scratch array",
                      static_cast<unsigned long long>(n), static_cast<unsigned long long>(EMMY_NOALLOC_MAX_ELEMENTS),
                      EMMY_NOALLOC_SCRATCH_BYTES);
    if (dev < 0 || dev >= 64) return report(EMMY_ERR_INVALID, "emmy_sum_f32_noalloc: bad device %d", dev);
    int prev_dev = 0;
    cudaError_t e = cudaGetDevice(&prev_dev);
    if (e != cudaSuccess) return report(EMMY_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if ((e = cudaSetDevice(dev)) != cudaSuccess)
        return report(EMMY_ERR_CUDA, "cudaSetDevice(%d): %s", dev, cudaGetErrorString(e));
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_ptr[dev]) {
            e = cudaGetSymbolAddress(&g_scratch_ptr[dev], g_noalloc_scratch);
            if (e != cudaSuccess) {
                g_scratch_ptr[dev] = nullptr;
                cudaSetDevice(prev_dev);
                return report(EMMY_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
            }
        }
        scratch = g_scratch_ptr[dev];
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint64_t chunk = kMinChunk;
    uint64_t nchunks = n ? (n + chunk - 1) / chunk : 1;
    const uint64_t target = static_cast<uint64_t>(kSms) * kBlocksPerSm;
    if (nchunks > target) {
        chunk = (n + target - 1) / target;
        chunk = (chunk + 1023) / 1024 * 1024;
        nchunks = (n + chunk - 1) / chunk;
    }
    int rc = EMMY_OK;
    e = cudaMemsetAsync(static_cast<unsigned char *>(scratch) + kCounterOffset, 0, sizeof(unsigned int), s);
    if (e != cudaSuccess) {
        rc = report(EMMY_ERR_CUDA, "clearing the arrival counter: %s", cudaGetErrorString(e));
    } else {
        const unsigned grid = static_cast<unsigned>(nchunks < target ? nchunks : target);
        noalloc_sum_kernel<<<grid, kThreads, 0, s>>>(x, n, chunk, static_cast<uint32_t>(nchunks), out,
                                                     static_cast<unsigned char *>(scratch));
        e = cudaGetLastError();
        if (e != cudaSuccess) rc = report(EMMY_ERR_CUDA, "launch: %s", cudaGetErrorString(e));
    }
    cudaSetDevice(prev_dev);
    return rc;
}

namespace {
int report(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return emmy_record_error(code, buf);
}
}  // namespace
