// Device side of the cross-GPU combine over NVLink peer memory.
//
// Every GPU of an exchange group owns one small buffer (emmy_xchg_create),
// mapped into every other GPU through CUDA IPC.  A combine of up to
// EMMY_XCHG_MAX_VALUES floats per GPU goes:
//
//   1. publish: for every rank r and value i, one 64-bit store of
//      (epoch << 32 | bits of value i) into word [parity][i][my rank] of r's
//      buffer.  The epoch and the value travel in one aligned 8-byte store,
//      so a reader never sees a new epoch with an old value;
//   2. wait (bounded by %globaltimer) until every word [parity][i][r] of this
//      GPU's own buffer carries this call's epoch;
//   3. the caller combines the gathered values in rank order, so every GPU
//      gets the same bits.
//
// parity = epoch & 1.  A GPU can be at most one call ahead of any other (it
// cannot finish call e+1 before every GPU has published e+1, which each does
// only after finishing call e), so call e+1 writes the other parity than a
// slower GPU may still be reading for call e.  That argument needs every GPU
// to finish every call; so a wait that runs out sets this GPU's FAILED word,
// and a GPU with FAILED set publishes nothing more and returns at once from
// every later call, until the host resets the group (emmy_xchg_reset, on
// every rank, with no call in flight anywhere).  A failed call leaves NaN in
// its outputs and bit 0 in the STATUS word.

#ifndef EMMY_XCHG_DEV_CUH
#define EMMY_XCHG_DEV_CUH

#include <stdint.h>

#define EMMY_XCHG_MAX_RANKS_DEV 8
#define EMMY_XCHG_MAX_VALUES 4
// buffer layout, bytes
#define EMMY_XCHG_STATUS_OFF 128u
#define EMMY_XCHG_FAILED_OFF 132u
#define EMMY_XCHG_WORDS_OFF 256u
#define EMMY_XCHG_BUFFER_BYTES 1024u

// Kernel parameter of a combining launch (passed by value).
struct EmmyXchgArgs {
    unsigned long long peer[EMMY_XCHG_MAX_RANKS_DEV];  // every rank's buffer, mapped here (own one included)
    unsigned long long local;                          // this GPU's buffer
    unsigned int rank, nranks, epoch, reserved;
    unsigned long long timeout_ns;
};

#ifdef __CUDACC__

__device__ __forceinline__ uint64_t emmy_xchg_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void emmy_xchg_store(unsigned long long addr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" :: "l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t emmy_xchg_load(unsigned long long addr) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long emmy_xchg_word(unsigned long long base, uint32_t par, int i, uint32_t r) {
    return base + EMMY_XCHG_WORDS_OFF + ((par * EMMY_XCHG_MAX_VALUES + i) * EMMY_XCHG_MAX_RANKS_DEV + r) * 8u;
}

// One thread: publish vals[0..n), gather every rank's into got[i * nranks + r].
// Returns false (and gathers nothing) when the group has failed or a peer did
// not arrive within the timeout.
static __device__ bool emmy_xchg_exchange(const EmmyXchgArgs &x, const float *vals, int n, float *got) {
    volatile uint32_t *failed = reinterpret_cast<volatile uint32_t *>(x.local + EMMY_XCHG_FAILED_OFF);
    uint32_t *status = reinterpret_cast<uint32_t *>(x.local + EMMY_XCHG_STATUS_OFF);
    if (*failed) {
        atomicOr(status, 1u);
        return false;
    }
    const uint32_t par = x.epoch & 1u;
    for (uint32_t r = 0; r < x.nranks; ++r)
        for (int i = 0; i < n; ++i)
            emmy_xchg_store(emmy_xchg_word(x.peer[r], par, i, x.rank),
                            (static_cast<uint64_t>(x.epoch) << 32) | __float_as_uint(vals[i]));
    const uint64_t t0 = emmy_xchg_now_ns();
    for (uint32_t r = 0; r < x.nranks; ++r) {
        for (int i = 0; i < n; ++i) {
            uint64_t w = emmy_xchg_load(emmy_xchg_word(x.local, par, i, r));
            while (static_cast<uint32_t>(w >> 32) != x.epoch) {
                if (emmy_xchg_now_ns() - t0 > x.timeout_ns) {
                    *failed = 1u;
                    __threadfence_system();
                    atomicOr(status, 1u);
                    return false;
                }
                __nanosleep(32);
                w = emmy_xchg_load(emmy_xchg_word(x.local, par, i, r));
            }
            got[i * x.nranks + r] = __uint_as_float(static_cast<uint32_t>(w));
        }
    }
    return true;
}

#endif  // __CUDACC__
#endif  // EMMY_XCHG_DEV_CUH
