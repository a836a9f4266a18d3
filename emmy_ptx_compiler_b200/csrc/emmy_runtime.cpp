// libemmy_b200: module loading, launching, host-buffer runs, timing and NCCL
// collectives behind the C ABI declared in include/emmy_b200.h.
//
// The CUDA driver and NCCL are opened with dlopen on first use, so the
// library loads (and its symbols can be inspected) on machines without a GPU
// driver.  Every entry point returns a status code and records a message
// for emmy_last_error(); nothing aborts.

#include "emmy_b200.h"
#include "emmy_launch_record.h"

#include <cuda.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace {

// ------------------------------------------------------------------ errors

thread_local std::string g_err;
thread_local int g_err_code = EMMY_OK;

int fail(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    g_err_code = code;
    return code;
}

// ------------------------------------------------------------------ driver table

struct Driver {
    void *lib = nullptr;
    bool ok = false;
#define EMMY_DRV(name) decltype(&::name) name = nullptr;
    EMMY_DRV(cuInit)
    EMMY_DRV(cuDeviceGetCount)
    EMMY_DRV(cuDeviceGet)
    EMMY_DRV(cuDeviceGetAttribute)
    EMMY_DRV(cuOccupancyMaxActiveBlocksPerMultiprocessor)
    EMMY_DRV(cuDevicePrimaryCtxRetain)
    EMMY_DRV(cuCtxSetCurrent)
    EMMY_DRV(cuCtxSynchronize)
    EMMY_DRV(cuModuleLoadDataEx)
    EMMY_DRV(cuModuleUnload)
    EMMY_DRV(cuModuleGetFunction)
    EMMY_DRV(cuModuleGetGlobal)
    EMMY_DRV(cuFuncSetAttribute)
    EMMY_DRV(cuFuncGetParamInfo)
    EMMY_DRV(cuLaunchKernel)
    EMMY_DRV(cuLaunchKernelEx)
    EMMY_DRV(cuMemAlloc)
    EMMY_DRV(cuMemFree)
    EMMY_DRV(cuMemAllocHost)
    EMMY_DRV(cuMemFreeHost)
    EMMY_DRV(cuMemHostGetDevicePointer)
    EMMY_DRV(cuMemcpyHtoD)
    EMMY_DRV(cuMemcpyDtoH)
    EMMY_DRV(cuMemcpyHtoDAsync)
    EMMY_DRV(cuMemcpyDtoHAsync)
    EMMY_DRV(cuMemsetD8Async)
    EMMY_DRV(cuStreamQuery)
    EMMY_DRV(cuStreamCreate)
    EMMY_DRV(cuStreamDestroy)
    EMMY_DRV(cuStreamWaitEvent)
    EMMY_DRV(cuStreamSynchronize)
    EMMY_DRV(cuEventCreate)
    EMMY_DRV(cuEventRecord)
    EMMY_DRV(cuEventSynchronize)
    EMMY_DRV(cuEventElapsedTime)
    EMMY_DRV(cuEventDestroy)
    EMMY_DRV(cuGetErrorString)
    EMMY_DRV(cuTensorMapEncodeTiled)
    EMMY_DRV(cuStreamBeginCapture)
    EMMY_DRV(cuStreamEndCapture)
    EMMY_DRV(cuGraphInstantiateWithFlags)
    EMMY_DRV(cuGraphLaunch)
    EMMY_DRV(cuGraphExecDestroy)
    EMMY_DRV(cuGraphDestroy)
#undef EMMY_DRV
};

Driver g_drv;
std::mutex g_mu;
std::vector<CUcontext> g_ctx;  // primary context per device
bool g_init = false;

typedef CUresult (*GetProcAddressFn)(const char *, void **, int, cuuint64_t,
                                     CUdriverProcAddressQueryResult *);

int load_driver() {
    if (g_drv.ok) return EMMY_OK;
    if (!g_drv.lib) g_drv.lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (!g_drv.lib) return fail(EMMY_ERR_NO_DRIVER, "cannot open libcuda.so.1: %s", dlerror());
    auto gpa = reinterpret_cast<GetProcAddressFn>(dlsym(g_drv.lib, "cuGetProcAddress_v2"));
    if (!gpa) return fail(EMMY_ERR_NO_DRIVER, "libcuda.so.1 has no cuGetProcAddress_v2");
    bool missing = false;
    std::string which;
    auto get = [&](const char *name, void **slot, bool required) {
        CUdriverProcAddressQueryResult st;
        if (gpa(name, slot, 12090, CU_GET_PROC_ADDRESS_DEFAULT, &st) != CUDA_SUCCESS || !*slot) {
            *slot = nullptr;
            if (required) {
                missing = true;
                which += std::string(" ") + name;
            }
        }
    };
#define EMMY_GET(name, req) get(#name, reinterpret_cast<void **>(&g_drv.name), req);
    EMMY_GET(cuInit, true)
    EMMY_GET(cuDeviceGetCount, true)
    EMMY_GET(cuDeviceGet, true)
    EMMY_GET(cuDeviceGetAttribute, true)
    EMMY_GET(cuOccupancyMaxActiveBlocksPerMultiprocessor, true)
    EMMY_GET(cuDevicePrimaryCtxRetain, true)
    EMMY_GET(cuCtxSetCurrent, true)
    EMMY_GET(cuCtxSynchronize, true)
    EMMY_GET(cuModuleLoadDataEx, true)
    EMMY_GET(cuModuleUnload, true)
    EMMY_GET(cuModuleGetFunction, true)
    EMMY_GET(cuModuleGetGlobal, true)
    EMMY_GET(cuFuncSetAttribute, true)
    EMMY_GET(cuFuncGetParamInfo, false)
    EMMY_GET(cuLaunchKernel, true)
    EMMY_GET(cuLaunchKernelEx, false)
    EMMY_GET(cuMemAlloc, true)
    EMMY_GET(cuMemFree, true)
    EMMY_GET(cuMemAllocHost, true)
    EMMY_GET(cuMemFreeHost, true)
    EMMY_GET(cuMemHostGetDevicePointer, false)
    EMMY_GET(cuMemcpyHtoD, true)
    EMMY_GET(cuMemcpyDtoH, true)
    EMMY_GET(cuMemcpyHtoDAsync, true)
    EMMY_GET(cuMemcpyDtoHAsync, true)
    EMMY_GET(cuMemsetD8Async, true)
    EMMY_GET(cuStreamQuery, true)
    EMMY_GET(cuStreamCreate, true)
    EMMY_GET(cuStreamDestroy, true)
    EMMY_GET(cuStreamWaitEvent, true)
    EMMY_GET(cuStreamSynchronize, true)
    EMMY_GET(cuEventCreate, true)
    EMMY_GET(cuEventRecord, true)
    EMMY_GET(cuEventSynchronize, true)
    EMMY_GET(cuEventElapsedTime, true)
    EMMY_GET(cuEventDestroy, true)
    EMMY_GET(cuGetErrorString, true)
    EMMY_GET(cuTensorMapEncodeTiled, false)
    EMMY_GET(cuStreamBeginCapture, false)
    EMMY_GET(cuStreamEndCapture, false)
    EMMY_GET(cuGraphInstantiateWithFlags, false)
    EMMY_GET(cuGraphLaunch, false)
    EMMY_GET(cuGraphExecDestroy, false)
    EMMY_GET(cuGraphDestroy, false)
#undef EMMY_GET
    if (missing) return fail(EMMY_ERR_NO_DRIVER, "driver lacks:%s", which.c_str());
    g_drv.ok = true;
    return EMMY_OK;
}

int cu_fail(CUresult r, const char *what) {
    const char *s = nullptr;
    if (g_drv.cuGetErrorString) g_drv.cuGetErrorString(r, &s);
    return fail(EMMY_ERR_CUDA, "%s failed: %s (%d)", what, s ? s : "?", static_cast<int>(r));
}

#define CU(call, what)                                      \
    do {                                                    \
        CUresult _r = (call);                               \
        if (_r != CUDA_SUCCESS) return cu_fail(_r, what);   \
    } while (0)

int set_device(int dev) {
    if (!g_init) return fail(EMMY_ERR_NOT_INIT, "emmy_init has not been called");
    if (dev < 0 || dev >= static_cast<int>(g_ctx.size()) || !g_ctx[dev])
        return fail(EMMY_ERR_NOT_FOUND, "device %d is not initialised", dev);
    CU(g_drv.cuCtxSetCurrent(g_ctx[dev]), "cuCtxSetCurrent");
    return EMMY_OK;
}

}  // namespace

// ------------------------------------------------------------------ modules

struct emmy_module {
    int dev = 0;
    CUmodule mod = nullptr;
    CUfunction fn = nullptr;
    CUfunction fn_dropin = nullptr;  // the arg_order-only entry when fn is its <entry>__emmy twin
    CUfunction fn_xchg = nullptr;    // <entry>__xchg: the reduction with the cross-GPU combine
    EmmyLaunchRecord rec{};
    bool has_rec = false;
    CUdeviceptr status = 0;
    std::vector<size_t> param_size;  // from cuFuncGetParamInfo (may be empty)
    // tensor-map cache: encoded for these source pointers
    std::vector<CUtensorMap> tmaps;
    std::vector<uint64_t> tmap_src;
    std::vector<uint64_t> tmap_rows;
    // emmy_run_host device buffers
    std::vector<CUdeviceptr> dbuf;
    std::vector<size_t> dbuf_bytes;
    // emmy_run_host chunk pipeline: copy-in and copy-out streams, one event pair per chunk
    CUstream h2d = nullptr, d2h = nullptr;
    std::vector<CUevent> ev_in, ev_out;
    CUevent ev_whole = nullptr, ev_start = nullptr;
    // largest dynamic shared memory the function may take (48 KiB unless raised)
    uint32_t dyn_attr = 48 * 1024;
    // emmy_run_host small-payload path: pinned host memory the kernel reads and writes directly
    void *zc_host = nullptr;
    CUdeviceptr zc_dev = 0;
    size_t zc_bytes = 0;
};

namespace {

bool has_range(const emmy_module *m);

// The tensor maps of a launch over units [rb, re).  A map over a streamed parameter (one that
// holds only its units' bytes in a sharded launch) starts at unit rb and spans re - rb units, so
// the TMA unit is never given an address outside the caller's buffer; the kernels address such
// maps relative to their first unit.
int encode_tmaps(emmy_module *m, const uint64_t *args, int nargs, uint64_t rb, uint64_t re) {
    const uint32_t n = m->has_rec ? m->rec.ntmaps : 0;
    if (n == 0) return EMMY_OK;
    if (!g_drv.cuTensorMapEncodeTiled)
        return fail(EMMY_ERR_NO_DRIVER, "driver lacks cuTensorMapEncodeTiled (needed by the GEMM family)");
    m->tmaps.resize(n);
    m->tmap_src.resize(n, ~0ull);
    m->tmap_rows.resize(n, ~0ull);
    for (uint32_t i = 0; i < n; ++i) {
        const EmmyTmapSpec &t = m->rec.tmaps[i];
        if (t.src_param >= static_cast<uint32_t>(nargs) || t.rank < 1 || t.rank > 5)
            return fail(EMMY_ERR_INVALID, "tensor map %u reads parameter %u of %d", i, t.src_param, nargs);
        uint64_t base = args[t.src_param];
        uint64_t rows = t.dims[t.rank - 1];
        const uint64_t unit_bytes = has_range(m) && t.src_param < EMMY_LR_MAX_PARAMS ? m->rec.range_bytes[t.src_param] : 0;
        if (unit_bytes) {
            if (rows != m->rec.range_total)
                return fail(EMMY_ERR_INVALID, "tensor map %u: outer extent %llu is not the unit count %llu", i,
                            (unsigned long long)rows, (unsigned long long)m->rec.range_total);
            base += rb * unit_bytes;
            rows = re - rb;
        }
        if (m->tmap_src[i] == base && m->tmap_rows[i] == rows) continue;
        if (base & 15ull) return fail(EMMY_ERR_INVALID, "TMA operand %u is not 16-byte aligned", t.src_param);
        cuuint64_t dims[5], strides[4];
        cuuint32_t box[5], estr[5];
        for (uint32_t d = 0; d < t.rank; ++d) {
            dims[d] = t.dims[d];
            box[d] = t.box[d];
            estr[d] = 1;
        }
        dims[t.rank - 1] = rows;
        for (uint32_t d = 0; d + 1 < t.rank; ++d) strides[d] = t.strides[d];
        CUresult r = g_drv.cuTensorMapEncodeTiled(
            &m->tmaps[i], static_cast<CUtensorMapDataType>(t.dtype), t.rank,
            reinterpret_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            static_cast<CUtensorMapSwizzle>(t.swizzle), static_cast<CUtensorMapL2promotion>(t.l2_promotion),
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cu_fail(r, "cuTensorMapEncodeTiled");
        m->tmap_src[i] = base;
        m->tmap_rows[i] = rows;
    }
    return EMMY_OK;
}

bool has_range(const emmy_module *m) { return m->has_rec && (m->rec.flags & EMMY_LR_RANGE); }

int launch_locked(emmy_module *m, const uint64_t *args, int nargs, const uint32_t *grid,
                  const uint32_t *block, uint64_t stream, uint64_t rbegin = 0, uint64_t rend = ~0ull,
                  int64_t dyn_override = -1) {
    int rc = set_device(m->dev);
    if (rc) return rc;
    uint32_t g[3], b[3], smem = 0;
    if (grid && block) {
        for (int i = 0; i < 3; ++i) {
            g[i] = grid[i] ? grid[i] : 1;
            b[i] = block[i] ? block[i] : 1;
        }
        smem = m->has_rec ? m->rec.dyn_smem : 0;
        if (dyn_override >= 0) {
            smem = static_cast<uint32_t>(dyn_override);
            if (smem > m->dyn_attr) {
                CU(g_drv.cuFuncSetAttribute(m->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                            static_cast<int>(smem)),
                   "cuFuncSetAttribute (dynamic shared memory)");
                m->dyn_attr = smem;
            }
        }
    } else if (m->has_rec) {
        for (int i = 0; i < 3; ++i) {
            g[i] = m->rec.grid[i];
            b[i] = m->rec.block[i];
        }
        smem = m->rec.dyn_smem;
    } else {
        return fail(EMMY_ERR_INVALID, "module has no launch record: pass grid and block");
    }
    if (m->has_rec && static_cast<uint32_t>(nargs) != m->rec.nparams)
        return fail(EMMY_ERR_INVALID, "entry takes %u parameters, got %d", m->rec.nparams, nargs);
    const size_t ntm = m->has_rec ? m->rec.ntmaps : 0;
    const bool ranged = has_range(m);
    uint64_t range[2] = {rbegin, rend == ~0ull && ranged ? m->rec.range_total : rend};
    if (ranged) {
        const uint64_t al = m->rec.range_align ? m->rec.range_align : 1;
        if (range[0] > range[1] || range[1] > m->rec.range_total || range[0] % al ||
            (range[1] % al && range[1] != m->rec.range_total))
            return fail(EMMY_ERR_INVALID, "unit range [%llu, %llu) is not within [0, %llu) in steps of %llu",
                        (unsigned long long)range[0], (unsigned long long)range[1],
                        (unsigned long long)m->rec.range_total, (unsigned long long)al);
        if (range[0] == range[1]) return EMMY_OK;
        if (!(grid && block) && (m->rec.flags & EMMY_LR_GRID_UNITS)) {
            const uint64_t per_cta = m->rec.grid_quantum ? m->rec.grid_quantum : 1;
            const uint64_t need = (range[1] - range[0] + per_cta - 1) / per_cta;
            if (need < g[0]) g[0] = static_cast<uint32_t>(need);
        }
    }
    if ((rc = encode_tmaps(m, args, nargs, ranged ? range[0] : 0, ranged ? range[1] : 0))) return rc;
    // fixed-size parameter tables: a launch allocates nothing on the host
    constexpr int kMaxArgs = 64;
    if (nargs < 0 || nargs > kMaxArgs) return fail(EMMY_ERR_INVALID, "%d parameters (at most %d)", nargs, kMaxArgs);
    void *kp[kMaxArgs + EMMY_LR_MAX_TMAPS + 2];
    uint32_t narrow[kMaxArgs];
    for (int i = 0; i < nargs; ++i) {
        size_t sz = 8;
        if (m->has_rec) sz = m->rec.param_kind[i] == EMMY_PARAM_PTR ? 8 : 4;
        else if (i < static_cast<int>(m->param_size.size())) sz = m->param_size[i];
        if (sz == 4) {
            narrow[i] = static_cast<uint32_t>(args[i]);
            kp[i] = &narrow[i];
        } else if (sz == 8) {
            kp[i] = const_cast<uint64_t *>(&args[i]);
        } else {
            return fail(EMMY_ERR_INVALID, "parameter %d has unsupported size %zu", i, sz);
        }
    }
    for (size_t i = 0; i < ntm; ++i) kp[static_cast<size_t>(nargs) + i] = &m->tmaps[i];
    if (ranged) {
        kp[static_cast<size_t>(nargs) + ntm] = &range[0];
        kp[static_cast<size_t>(nargs) + ntm + 1] = &range[1];
    }
    const bool cluster = m->has_rec && (m->rec.flags & 0xFFu) > 1u;
    const bool coop = m->has_rec && (m->rec.flags & EMMY_LR_COOPERATIVE);
    if (cluster || coop) {
        if (!g_drv.cuLaunchKernelEx) return fail(EMMY_ERR_NO_DRIVER, "driver lacks cuLaunchKernelEx");
        CUlaunchAttribute attr[2];
        unsigned nattr = 0;
        if (cluster) {
            attr[nattr].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
            attr[nattr].value.clusterDim.x = m->rec.flags & 0xFFu;
            attr[nattr].value.clusterDim.y = 1;
            attr[nattr].value.clusterDim.z = 1;
            ++nattr;
        }
        if (coop) {
            // every CTA resident at once, or the launch fails (the CTAs wait on one another)
            attr[nattr].id = CU_LAUNCH_ATTRIBUTE_COOPERATIVE;
            attr[nattr].value.cooperative = 1;
            ++nattr;
        }
        CUlaunchConfig cfg{};
        cfg.gridDimX = g[0];
        cfg.gridDimY = g[1];
        cfg.gridDimZ = g[2];
        cfg.blockDimX = b[0];
        cfg.blockDimY = b[1];
        cfg.blockDimZ = b[2];
        cfg.sharedMemBytes = smem;
        cfg.hStream = reinterpret_cast<CUstream>(stream);
        cfg.attrs = attr;
        cfg.numAttrs = nattr;
        CU(g_drv.cuLaunchKernelEx(&cfg, m->fn, kp, nullptr), "cuLaunchKernelEx");
    } else {
        CU(g_drv.cuLaunchKernel(m->fn, g[0], g[1], g[2], b[0], b[1], b[2], smem,
                                reinterpret_cast<CUstream>(stream), kp, nullptr),
           "cuLaunchKernel");
    }
    return EMMY_OK;
}

}  // namespace

// emmy_xchg.cu: the next combining call's kernel parameter (struct EmmyXchgArgs of
// emmy_xchg_dev.cuh, kXchgArgsBytes bytes) for exchange group x on device dev.
extern "C" int emmy_xchg_fill_args(emmy_xchg_t x, int dev, int timeout_ms, void *args, size_t bytes);
constexpr size_t kXchgArgsBytes = 8 * 8 + 8 + 4 * 4 + 8;

// Lets other translation units of the library report through emmy_last_error.
extern "C" __attribute__((visibility("hidden"))) int emmy_record_error(int code, const char *msg) {
    return fail(code, "%s", msg);
}

extern "C" {

const char *emmy_version(void) { return "emmy_b200 1.0 (sm_100a)"; }

int emmy_last_error(char *buf, size_t len) {
    if (buf && len) {
        std::strncpy(buf, g_err.c_str(), len - 1);
        buf[len - 1] = '\0';
    }
    return g_err_code;
}

int emmy_init(int ndev) {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = load_driver();
    if (rc) return rc;
    CUresult r = g_drv.cuInit(0);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuInit");
    int count = 0;
    CU(g_drv.cuDeviceGetCount(&count), "cuDeviceGetCount");
    if (count <= 0) return fail(EMMY_ERR_NOT_FOUND, "no CUDA devices");
    const int n = (ndev <= 0 || ndev > count) ? count : ndev;
    if (static_cast<int>(g_ctx.size()) < n) g_ctx.resize(n, nullptr);
    for (int i = 0; i < n; ++i) {
        if (g_ctx[i]) continue;
        CUdevice d;
        CU(g_drv.cuDeviceGet(&d, i), "cuDeviceGet");
        CU(g_drv.cuDevicePrimaryCtxRetain(&g_ctx[i], d), "cuDevicePrimaryCtxRetain");
    }
    g_init = true;
    return EMMY_OK;
}

int emmy_device_count(int *count) {
    if (!count) return fail(EMMY_ERR_INVALID, "count is NULL");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = load_driver();
    if (rc) return rc;
    CUresult r = g_drv.cuInit(0);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuInit");
    CU(g_drv.cuDeviceGetCount(count), "cuDeviceGetCount");
    return EMMY_OK;
}

int emmy_load(int dev, const void *image, size_t len, const char *entry, emmy_module_t *out) {
    if (!image || !len || !entry || !out) return fail(EMMY_ERR_INVALID, "emmy_load: NULL argument");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc) return rc;
    // PTX must be NUL-terminated; cubin (ELF) is passed through.
    std::vector<char> buf(static_cast<const char *>(image), static_cast<const char *>(image) + len);
    const bool elf = len >= 4 && std::memcmp(image, "\x7f" "ELF", 4) == 0;
    if (!elf) buf.push_back('\0');
    char log[8192] = {0};
    CUjit_option opts[2] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
    void *vals[2] = {log, reinterpret_cast<void *>(static_cast<uintptr_t>(sizeof log))};
    auto *m = new emmy_module();
    m->dev = dev;
    CUresult r = g_drv.cuModuleLoadDataEx(&m->mod, buf.data(), 2, opts, vals);
    if (r != CUDA_SUCCESS) {
        delete m;
        const char *s = nullptr;
        g_drv.cuGetErrorString(r, &s);
        return fail(EMMY_ERR_CUDA, "cuModuleLoadDataEx: %s: %s", s ? s : "?", log);
    }
    r = g_drv.cuModuleGetFunction(&m->fn, m->mod, entry);
    if (r != CUDA_SUCCESS) {
        g_drv.cuModuleUnload(m->mod);
        delete m;
        return fail(EMMY_ERR_NOT_FOUND, "entry '%s' not found in module", entry);
    }
    {
        // modules of our compiler whose fast kernel takes more than the arg_order
        // parameters (a unit range, tensor maps) export it as <entry>__emmy beside
        // the drop-in <entry>; the library launches the fast one
        char native[512];
        if (std::snprintf(native, sizeof native, "%s__emmy", entry) < static_cast<int>(sizeof native)) {
            CUfunction fast = nullptr;
            if (g_drv.cuModuleGetFunction(&fast, m->mod, native) == CUDA_SUCCESS && fast) {
                m->fn_dropin = m->fn;
                m->fn = fast;
            }
        }
        if (std::snprintf(native, sizeof native, "%s__xchg", entry) < static_cast<int>(sizeof native)) {
            CUfunction xf = nullptr;
            if (g_drv.cuModuleGetFunction(&xf, m->mod, native) == CUDA_SUCCESS) m->fn_xchg = xf;
        }
    }
    CUdeviceptr rec_ptr = 0;
    size_t rec_bytes = 0;
    if (g_drv.cuModuleGetGlobal(&rec_ptr, &rec_bytes, m->mod, "emmy_launch_record") == CUDA_SUCCESS &&
        rec_bytes == sizeof(EmmyLaunchRecord)) {
        r = g_drv.cuMemcpyDtoH(&m->rec, rec_ptr, sizeof m->rec);
        if (r != CUDA_SUCCESS) {
            g_drv.cuModuleUnload(m->mod);
            delete m;
            return cu_fail(r, "reading emmy_launch_record");
        }
        if (m->rec.magic == EMMY_LR_MAGIC && m->rec.version == EMMY_LR_VERSION) {
            if (m->rec.nparams > EMMY_LR_MAX_PARAMS || m->rec.ntmaps > EMMY_LR_MAX_TMAPS) {
                g_drv.cuModuleUnload(m->mod);
                delete m;
                return fail(EMMY_ERR_INVALID, "launch record lists %u parameters and %u tensor maps (at most %d, %d)",
                            m->rec.nparams, m->rec.ntmaps, EMMY_LR_MAX_PARAMS, EMMY_LR_MAX_TMAPS);
            }
            m->has_rec = true;
        }
    }
    size_t st_bytes = 0;
    if (g_drv.cuModuleGetGlobal(&m->status, &st_bytes, m->mod, "emmy_status") != CUDA_SUCCESS)
        m->status = 0;
    if (g_drv.cuFuncGetParamInfo) {
        for (size_t i = 0; i < 256; ++i) {
            size_t off = 0, sz = 0;
            if (g_drv.cuFuncGetParamInfo(m->fn, i, &off, &sz) != CUDA_SUCCESS) break;
            m->param_size.push_back(sz);
        }
    }
    if (m->has_rec) {
        const size_t want = m->rec.nparams + m->rec.ntmaps + ((m->rec.flags & EMMY_LR_RANGE) ? 2 : 0);
        if (!m->param_size.empty() && m->param_size.size() != want) {
            g_drv.cuModuleUnload(m->mod);
            delete m;
            return fail(EMMY_ERR_INVALID, "entry has %zu parameters, launch record says %zu",
                        m->param_size.size(), want);
        }
        if (m->rec.dyn_smem > 48 * 1024) {
            m->dyn_attr = m->rec.dyn_smem;
            r = g_drv.cuFuncSetAttribute(m->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                         static_cast<int>(m->rec.dyn_smem));
            if (r != CUDA_SUCCESS) {
                g_drv.cuModuleUnload(m->mod);
                delete m;
                return cu_fail(r, "cuFuncSetAttribute(max dynamic smem)");
            }
        }
        if (m->rec.flags & EMMY_LR_FILL_GRID) {
            // grid = waves x (resident CTAs per SM for this build) x SMs, in whole quanta
            CUdevice d = 0;
            int nsm = 0, occ = 0;
            const int threads = static_cast<int>(m->rec.block[0] * m->rec.block[1] * m->rec.block[2]);
            r = g_drv.cuDeviceGet(&d, dev);
            if (r == CUDA_SUCCESS) r = g_drv.cuDeviceGetAttribute(&nsm, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, d);
            if (r == CUDA_SUCCESS)
                r = g_drv.cuOccupancyMaxActiveBlocksPerMultiprocessor(&occ, m->fn, threads, m->rec.dyn_smem);
            if (r != CUDA_SUCCESS) {
                g_drv.cuModuleUnload(m->mod);
                delete m;
                return cu_fail(r, "sizing the grid from occupancy");
            }
            const uint64_t waves = m->rec.grid[0] ? m->rec.grid[0] : 1u;
            const uint64_t q = m->rec.grid_quantum ? m->rec.grid_quantum : 1u;
            uint64_t g = waves * static_cast<uint64_t>(occ > 0 ? occ : 1) * static_cast<uint64_t>(nsm > 0 ? nsm : 1);
            g = g / q * q;
            if (g == 0) g = q;
            if (g > 0x7FFFFFFFu) g = 0x7FFFFFFFu / q * q;
            m->rec.grid[0] = static_cast<uint32_t>(g);
        }
    }
    *out = m;
    return EMMY_OK;
}

int emmy_unload(emmy_module_t m) {
    if (!m) return EMMY_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(m->dev);
    if (rc) return rc;
    for (CUdeviceptr p : m->dbuf)
        if (p) g_drv.cuMemFree(p);
    for (CUevent e : m->ev_in) g_drv.cuEventDestroy(e);
    for (CUevent e : m->ev_out) g_drv.cuEventDestroy(e);
    if (m->ev_whole) g_drv.cuEventDestroy(m->ev_whole);
    if (m->ev_start) g_drv.cuEventDestroy(m->ev_start);
    if (m->h2d) g_drv.cuStreamDestroy(m->h2d);
    if (m->d2h) g_drv.cuStreamDestroy(m->d2h);
    if (m->zc_host) g_drv.cuMemFreeHost(m->zc_host);
    CUresult r = g_drv.cuModuleUnload(m->mod);
    delete m;
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuModuleUnload");
    return EMMY_OK;
}

int emmy_module_info(emmy_module_t m, uint32_t *family, uint32_t grid[3], uint32_t block[3],
                     uint32_t *dyn_smem, uint32_t *nparams) {
    if (!m) return fail(EMMY_ERR_INVALID, "module is NULL");
    if (family) *family = m->has_rec ? m->rec.family : 0;
    for (int i = 0; i < 3; ++i) {
        if (grid) grid[i] = m->has_rec ? m->rec.grid[i] : 0;
        if (block) block[i] = m->has_rec ? m->rec.block[i] : 0;
    }
    if (dyn_smem) *dyn_smem = m->has_rec ? m->rec.dyn_smem : 0;
    if (nparams)
        *nparams = m->has_rec ? m->rec.nparams : static_cast<uint32_t>(m->param_size.size());
    return EMMY_OK;
}

int emmy_launch(emmy_module_t m, const uint64_t *args, int nargs, const uint32_t *grid,
                const uint32_t *block, uint64_t stream) {
    if (!m || (nargs > 0 && !args)) return fail(EMMY_ERR_INVALID, "emmy_launch: NULL argument");
    std::lock_guard<std::mutex> lk(g_mu);
    return launch_locked(m, args, nargs, grid, block, stream);
}

int emmy_launch_ex(emmy_module_t m, const uint64_t *args, int nargs, const uint32_t *grid,
                   const uint32_t *block, uint32_t dyn_smem, uint64_t stream) {
    if (!m || (nargs > 0 && !args) || !grid || !block)
        return fail(EMMY_ERR_INVALID, "emmy_launch_ex: NULL argument (grid and block are required)");
    std::lock_guard<std::mutex> lk(g_mu);
    return launch_locked(m, args, nargs, grid, block, stream, 0, ~0ull, static_cast<int64_t>(dyn_smem));
}

int emmy_module_status(emmy_module_t m, uint32_t *status) {
    if (!m || !status) return fail(EMMY_ERR_INVALID, "emmy_module_status: NULL argument");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(m->dev);
    if (rc) return rc;
    *status = 0;
    if (!m->status) return EMMY_OK;
    CU(g_drv.cuCtxSynchronize(), "cuCtxSynchronize");
    CU(g_drv.cuMemcpyDtoH(status, m->status, sizeof(uint32_t)), "reading emmy_status");
    if (*status) {
        const uint32_t zero = 0;
        CU(g_drv.cuMemcpyHtoD(m->status, &zero, sizeof zero), "clearing emmy_status");
    }
    return EMMY_OK;
}

int emmy_sync(int dev, uint64_t stream, int timeout_ms) {
    {
        std::lock_guard<std::mutex> lk(g_mu);
        int rc = set_device(dev);
        if (rc) return rc;
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        CUresult r = g_drv.cuStreamQuery(reinterpret_cast<CUstream>(stream));
        if (r == CUDA_SUCCESS) return EMMY_OK;
        if (r != CUDA_ERROR_NOT_READY) return cu_fail(r, "cuStreamQuery");
        if (timeout_ms > 0) {
            const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                std::chrono::steady_clock::now() - t0);
            if (el.count() > timeout_ms)
                return fail(EMMY_ERR_TIMEOUT, "stream not idle after %d ms", timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int emmy_alloc(int dev, size_t bytes, uint64_t *dptr) {
    if (!dptr) return fail(EMMY_ERR_INVALID, "dptr is NULL");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc) return rc;
    CUdeviceptr p = 0;
    CU(g_drv.cuMemAlloc(&p, bytes ? bytes : 1), "cuMemAlloc");
    *dptr = p;
    return EMMY_OK;
}

int emmy_free(int dev, uint64_t dptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc) return rc;
    if (dptr) CU(g_drv.cuMemFree(dptr), "cuMemFree");
    return EMMY_OK;
}

int emmy_memcpy_htod(int dev, uint64_t dst, const void *src, size_t bytes, uint64_t stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc) return rc;
    CU(g_drv.cuMemcpyHtoDAsync(dst, src, bytes, reinterpret_cast<CUstream>(stream)), "cuMemcpyHtoDAsync");
    return EMMY_OK;
}

int emmy_memcpy_dtoh(int dev, void *dst, uint64_t src, size_t bytes, uint64_t stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc) return rc;
    CU(g_drv.cuMemcpyDtoHAsync(dst, src, bytes, reinterpret_cast<CUstream>(stream)), "cuMemcpyDtoHAsync");
    CU(g_drv.cuStreamSynchronize(reinterpret_cast<CUstream>(stream)), "cuStreamSynchronize");
    return EMMY_OK;
}

int emmy_memset_d8(int dev, uint64_t dst, uint8_t value, size_t bytes, uint64_t stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc) return rc;
    CU(g_drv.cuMemsetD8Async(dst, value, bytes, reinterpret_cast<CUstream>(stream)), "cuMemsetD8Async");
    return EMMY_OK;
}

int emmy_host_alloc(size_t bytes, void **ptr) {
    if (!ptr) return fail(EMMY_ERR_INVALID, "ptr is NULL");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(0);
    if (rc) return rc;
    CU(g_drv.cuMemAllocHost(ptr, bytes ? bytes : 1), "cuMemAllocHost");
    return EMMY_OK;
}

int emmy_host_free(void *ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(0);
    if (rc) return rc;
    if (ptr) CU(g_drv.cuMemFreeHost(ptr), "cuMemFreeHost");
    return EMMY_OK;
}

}  // extern "C"

namespace {

bool is_in(uint8_t r) { return r == EMMY_ROLE_IN || r == EMMY_ROLE_INOUT; }
bool is_out(uint8_t r) { return r == EMMY_ROLE_OUT || r == EMMY_ROLE_INOUT || r == EMMY_ROLE_OUT_ZEROED; }

// Bytes [lo, hi) of parameter i's unit range, clipped to the caller's buffer.
void unit_bytes(const emmy_module *m, int i, uint64_t b, uint64_t e, size_t have, size_t *lo, size_t *hi) {
    const uint64_t per = m->rec.range_bytes[i];
    *lo = static_cast<size_t>(std::min<uint64_t>(b * per, have));
    *hi = static_cast<size_t>(std::min<uint64_t>(e * per, have));
}

int ensure_pipeline(emmy_module *m, size_t nchunks) {
    if (!m->h2d) CU(g_drv.cuStreamCreate(&m->h2d, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
    if (!m->d2h) CU(g_drv.cuStreamCreate(&m->d2h, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
    if (!m->ev_whole) CU(g_drv.cuEventCreate(&m->ev_whole, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
    if (!m->ev_start) CU(g_drv.cuEventCreate(&m->ev_start, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
    while (m->ev_in.size() < nchunks) {
        CUevent a, b;
        CU(g_drv.cuEventCreate(&a, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
        CU(g_drv.cuEventCreate(&b, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
        m->ev_in.push_back(a);
        m->ev_out.push_back(b);
    }
    return EMMY_OK;
}

constexpr uint64_t kChunkBytesDefault = 64ull << 20;  // streamed bytes per pipeline chunk (in + out)
constexpr uint64_t kMaxPipelineChunks = 256;

// EMMY_PIPELINE_CHUNK_BYTES overrides the chunk size (bytes of streamed copies per chunk,
// at least 1 MiB) for callers that tune the copy pipeline to their host link.
uint64_t pipeline_chunk_bytes() {
    const char *v = std::getenv("EMMY_PIPELINE_CHUNK_BYTES");
    if (v && *v) {
        const unsigned long long b = std::strtoull(v, nullptr, 10);
        if (b >= (1ull << 20)) return b;
    }
    return kChunkBytesDefault;
}

// The chunk pipeline of emmy_run_host (caller holds g_mu, device is current).
int run_pipeline(emmy_module *m, void *const *host_ptrs, const size_t *bytes, const uint8_t *roles, int nargs,
                 uint64_t stream, std::vector<uint64_t> &args, uint64_t total, uint64_t align, uint64_t streamed,
                 uint64_t chunk_bytes) {
    CUstream s = reinterpret_cast<CUstream>(stream);
    int rc = EMMY_OK;
    // Unit ranges [b, e) flow through copy-in (h2d stream), the
    // kernel (`stream`) and copy-out (d2h stream), so chunk k's copy-in, chunk
    // k-1's kernel and chunk k-2's copy-out overlap, and both host-link
    // directions are busy at once.
    uint64_t nchunks = std::max<uint64_t>(2, std::min<uint64_t>(kMaxPipelineChunks / 2, streamed / chunk_bytes));
    uint64_t per = (total + nchunks - 1) / nchunks;
    per = (per + align - 1) / align * align;
    // Chunk boundaries (in units of `align`): the first chunks grow from per / 16 to per and the
    // last ones shrink back, so that the copy-in before the first kernel and the copy-out after
    // the last one (while one link direction idles) are short.
    std::vector<uint64_t> cut{0};
    {
        const uint64_t U = (total + align - 1) / align, P = std::max<uint64_t>(1, per / align);
        std::vector<uint64_t> ramp;
        uint64_t ramp_units = 0;
        for (uint64_t sz = std::max<uint64_t>(1, P / 16); sz < P; sz *= 2) {
            ramp.push_back(sz);
            ramp_units += sz;
        }
        if (U < 2 * ramp_units + 2 * P) {
            ramp.clear();
            ramp_units = 0;
        }
        uint64_t u = 0;
        for (uint64_t sz : ramp) cut.push_back((u += sz) * align);
        const uint64_t mid_end = U - ramp_units;
        while (u + P < mid_end) cut.push_back((u += P) * align);
        if (mid_end > u) cut.push_back((u = mid_end) * align);
        for (auto it = ramp.rbegin(); it != ramp.rend(); ++it) cut.push_back((u += *it) * align);
        cut.back() = total;   // the last unit may be partial
    }
    nchunks = cut.size() - 1;
    if ((rc = ensure_pipeline(m, nchunks))) return rc;
    CU(g_drv.cuEventRecord(m->ev_start, s), "cuEventRecord");
    CU(g_drv.cuStreamWaitEvent(m->h2d, m->ev_start, 0), "cuStreamWaitEvent");
    CU(g_drv.cuStreamWaitEvent(m->d2h, m->ev_start, 0), "cuStreamWaitEvent");
    for (int i = 0; i < nargs; ++i) {
        if (roles[i] == EMMY_ROLE_SCALAR) continue;
        if (is_in(roles[i]) && !m->rec.range_bytes[i])
            CU(g_drv.cuMemcpyHtoDAsync(m->dbuf[i], host_ptrs[i], bytes[i], m->h2d), "cuMemcpyHtoDAsync");
        if (roles[i] == EMMY_ROLE_OUT_ZEROED)
            CU(g_drv.cuMemsetD8Async(m->dbuf[i], 0, bytes[i], s), "cuMemsetD8Async");
    }
    CU(g_drv.cuEventRecord(m->ev_whole, m->h2d), "cuEventRecord");
    CU(g_drv.cuStreamWaitEvent(s, m->ev_whole, 0), "cuStreamWaitEvent");
    for (uint64_t k = 0; k < nchunks; ++k) {
        const uint64_t b = cut[k], e = cut[k + 1];
        for (int i = 0; i < nargs; ++i) {
            if (roles[i] == EMMY_ROLE_SCALAR || !is_in(roles[i]) || !m->rec.range_bytes[i]) continue;
            size_t lo, hi;
            unit_bytes(m, i, b, e, bytes[i], &lo, &hi);
            if (hi > lo)
                CU(g_drv.cuMemcpyHtoDAsync(m->dbuf[i] + lo, static_cast<const char *>(host_ptrs[i]) + lo, hi - lo,
                                           m->h2d),
                   "cuMemcpyHtoDAsync");
        }
        CU(g_drv.cuEventRecord(m->ev_in[k], m->h2d), "cuEventRecord");
        CU(g_drv.cuStreamWaitEvent(s, m->ev_in[k], 0), "cuStreamWaitEvent");
        if ((rc = launch_locked(m, args.data(), nargs, nullptr, nullptr, stream, b, e))) return rc;
        CU(g_drv.cuEventRecord(m->ev_out[k], s), "cuEventRecord");
        CU(g_drv.cuStreamWaitEvent(m->d2h, m->ev_out[k], 0), "cuStreamWaitEvent");
        for (int i = 0; i < nargs; ++i) {
            if (roles[i] == EMMY_ROLE_SCALAR || !is_out(roles[i]) || !m->rec.range_bytes[i]) continue;
            size_t lo, hi;
            unit_bytes(m, i, b, e, bytes[i], &lo, &hi);
            if (hi > lo)
                CU(g_drv.cuMemcpyDtoHAsync(static_cast<char *>(host_ptrs[i]) + lo, m->dbuf[i] + lo, hi - lo, m->d2h),
                   "cuMemcpyDtoHAsync");
        }
    }
    // outputs written whole by every launch leave after the last one (d2h already waits on it)
    for (int i = 0; i < nargs; ++i)
        if (roles[i] != EMMY_ROLE_SCALAR && is_out(roles[i]) && !m->rec.range_bytes[i])
            CU(g_drv.cuMemcpyDtoHAsync(host_ptrs[i], m->dbuf[i], bytes[i], m->d2h), "cuMemcpyDtoHAsync");
    CU(g_drv.cuStreamSynchronize(m->d2h), "cuStreamSynchronize");
    CU(g_drv.cuStreamSynchronize(s), "cuStreamSynchronize");
    CU(g_drv.cuStreamSynchronize(m->h2d), "cuStreamSynchronize");
    return EMMY_OK;
}

}  // namespace

extern "C" {

namespace {

constexpr size_t kMappedMaxBytes = 64 * 1024;
constexpr size_t kMappedAlign = 256;

// Problems of at most 64 KiB in all go through pinned host memory that the
// kernel reads and writes over PCIe itself: no copy engine round trips, which
// dominate at these sizes.  Only for families whose kernels touch their
// parameters with plain loads and stores (pointwise, row-fused): no atomics,
// tensor maps or async copies on host memory.
bool mapped_path_ok(const emmy_module *m, const size_t *bytes, const uint8_t *roles, int nargs) {
    if (!m->has_rec || m->rec.ntmaps != 0 || !g_drv.cuMemHostGetDevicePointer) return false;
    if (m->rec.family != EMMY_FAMILY_POINTWISE && m->rec.family != EMMY_FAMILY_ROWFUSED) return false;
    size_t total = 0;
    for (int i = 0; i < nargs; ++i) {
        if (roles[i] == EMMY_ROLE_SCALAR) continue;
        total = (total + kMappedAlign - 1) / kMappedAlign * kMappedAlign + bytes[i];
        if (total > kMappedMaxBytes) return false;
    }
    return nargs <= 64;
}

int run_host_mapped(emmy_module *m, void *const *host_ptrs, const size_t *bytes, const uint8_t *roles, int nargs,
                    uint64_t stream) {
    if (!m->zc_host) {
        CU(g_drv.cuMemAllocHost(&m->zc_host, kMappedMaxBytes), "cuMemAllocHost (run_host small path)");
        CUresult r = g_drv.cuMemHostGetDevicePointer(&m->zc_dev, m->zc_host, 0);
        if (r != CUDA_SUCCESS) {
            g_drv.cuMemFreeHost(m->zc_host);
            m->zc_host = nullptr;
            return cu_fail(r, "cuMemHostGetDevicePointer");
        }
        m->zc_bytes = kMappedMaxBytes;
    }
    uint64_t args[64];
    size_t offs[64];
    size_t off = 0;
    char *base = static_cast<char *>(m->zc_host);
    for (int i = 0; i < nargs; ++i) {
        if (roles[i] == EMMY_ROLE_SCALAR) {
            uint32_t v = 0;
            std::memcpy(&v, host_ptrs[i], 4);
            args[i] = v;
            continue;
        }
        off = (off + kMappedAlign - 1) / kMappedAlign * kMappedAlign;
        offs[i] = off;
        if (is_in(roles[i]))
            std::memcpy(base + off, host_ptrs[i], bytes[i]);
        else if (roles[i] == EMMY_ROLE_OUT_ZEROED)
            std::memset(base + off, 0, bytes[i]);
        args[i] = m->zc_dev + off;
        off += bytes[i];
    }
    int rc = launch_locked(m, args, nargs, nullptr, nullptr, stream);
    if (rc) return rc;
    CU(g_drv.cuStreamSynchronize(reinterpret_cast<CUstream>(stream)), "cuStreamSynchronize");
    for (int i = 0; i < nargs; ++i)
        if (roles[i] != EMMY_ROLE_SCALAR && is_out(roles[i])) std::memcpy(host_ptrs[i], base + offs[i], bytes[i]);
    return EMMY_OK;
}

}  // namespace

int emmy_run_host(emmy_module_t m, void *const *host_ptrs, const size_t *bytes, const uint8_t *roles,
                  int nargs, uint64_t stream) {
    if (!m || (nargs > 0 && (!host_ptrs || !bytes || !roles)))
        return fail(EMMY_ERR_INVALID, "emmy_run_host: NULL argument");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(m->dev);
    if (rc) return rc;
    if (mapped_path_ok(m, bytes, roles, nargs)) return run_host_mapped(m, host_ptrs, bytes, roles, nargs, stream);
    CUstream s = reinterpret_cast<CUstream>(stream);
    if (static_cast<int>(m->dbuf.size()) < nargs) {
        m->dbuf.resize(nargs, 0);
        m->dbuf_bytes.resize(nargs, 0);
    }
    std::vector<uint64_t> args(nargs);
    uint64_t streamed = 0;
    for (int i = 0; i < nargs; ++i) {
        if (roles[i] == EMMY_ROLE_SCALAR) {
            uint32_t v = 0;
            std::memcpy(&v, host_ptrs[i], 4);
            args[i] = v;
            continue;
        }
        if (m->dbuf_bytes[i] < bytes[i]) {
            if (m->dbuf[i]) g_drv.cuMemFree(m->dbuf[i]);
            m->dbuf[i] = 0;
            m->dbuf_bytes[i] = 0;
            CU(g_drv.cuMemAlloc(&m->dbuf[i], bytes[i] ? bytes[i] : 1), "cuMemAlloc (run_host)");
            m->dbuf_bytes[i] = bytes[i];
        }
        args[i] = m->dbuf[i];
        if (has_range(m) && i < EMMY_LR_MAX_PARAMS && m->rec.range_bytes[i]) streamed += bytes[i];
    }
    const uint64_t total = has_range(m) ? m->rec.range_total : 0;
    const uint64_t align = has_range(m) && m->rec.range_align ? m->rec.range_align : 1;
    const uint64_t chunk_bytes = pipeline_chunk_bytes();
    if (total < 2 * align || streamed < 2 * chunk_bytes) {
        // one launch: copy in, launch, copy out, all on `stream`
        for (int i = 0; i < nargs; ++i) {
            if (roles[i] == EMMY_ROLE_SCALAR) continue;
            if (is_in(roles[i]))
                CU(g_drv.cuMemcpyHtoDAsync(m->dbuf[i], host_ptrs[i], bytes[i], s), "cuMemcpyHtoDAsync");
            else if (roles[i] == EMMY_ROLE_OUT_ZEROED)
                CU(g_drv.cuMemsetD8Async(m->dbuf[i], 0, bytes[i], s), "cuMemsetD8Async");
        }
        if ((rc = launch_locked(m, args.data(), nargs, nullptr, nullptr, stream))) return rc;
        for (int i = 0; i < nargs; ++i)
            if (roles[i] != EMMY_ROLE_SCALAR && is_out(roles[i]))
                CU(g_drv.cuMemcpyDtoHAsync(host_ptrs[i], m->dbuf[i], bytes[i], s), "cuMemcpyDtoHAsync");
        CU(g_drv.cuStreamSynchronize(s), "cuStreamSynchronize");
        return EMMY_OK;
    }
    rc = run_pipeline(m, host_ptrs, bytes, roles, nargs, stream, args, total, align, streamed, chunk_bytes);
    if (rc) {
        // leave no copy or kernel of this call in flight on the module's buffers (best effort)
        g_drv.cuStreamSynchronize(m->h2d);
        g_drv.cuStreamSynchronize(s);
        g_drv.cuStreamSynchronize(m->d2h);
    }
    return rc;
}

int emmy_launch_range(emmy_module_t m, const uint64_t *args, int nargs, uint64_t begin, uint64_t end,
                      uint64_t stream) {
    if (!m || (nargs > 0 && !args)) return fail(EMMY_ERR_INVALID, "emmy_launch_range: NULL argument");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!has_range(m)) return fail(EMMY_ERR_INVALID, "module takes no unit range (launch record has no EMMY_LR_RANGE)");
    return launch_locked(m, args, nargs, nullptr, nullptr, stream, begin, end);
}

int emmy_launch_xchg(emmy_module_t m, const uint64_t *args, int nargs, emmy_xchg_t x, int timeout_ms,
                     uint64_t stream) {
    if (!m || !x || (nargs > 0 && !args)) return fail(EMMY_ERR_INVALID, "emmy_launch_xchg: NULL argument");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!m->fn_xchg || !m->has_rec)
        return fail(EMMY_ERR_INVALID, "module has no cross-GPU combine entry (only full-array reductions do)");
    if (static_cast<uint32_t>(nargs) != m->rec.nparams || nargs > EMMY_LR_MAX_PARAMS)
        return fail(EMMY_ERR_INVALID, "entry takes %u parameters, got %d", m->rec.nparams, nargs);
    int rc = set_device(m->dev);
    if (rc) return rc;
    alignas(16) unsigned char xargs[kXchgArgsBytes];
    if ((rc = emmy_xchg_fill_args(x, m->dev, timeout_ms, xargs, sizeof xargs))) return rc;
    void *kp[EMMY_LR_MAX_PARAMS + 1];
    uint32_t narrow[EMMY_LR_MAX_PARAMS];
    for (int i = 0; i < nargs; ++i) {
        if (m->rec.param_kind[i] == EMMY_PARAM_PTR) {
            kp[i] = const_cast<uint64_t *>(&args[i]);
        } else {
            narrow[i] = static_cast<uint32_t>(args[i]);
            kp[i] = &narrow[i];
        }
    }
    kp[nargs] = xargs;
    CU(g_drv.cuLaunchKernel(m->fn_xchg, m->rec.grid[0], m->rec.grid[1], m->rec.grid[2], m->rec.block[0],
                            m->rec.block[1], m->rec.block[2], m->rec.dyn_smem, reinterpret_cast<CUstream>(stream),
                            kp, nullptr),
       "cuLaunchKernel (cross-GPU combine)");
    return EMMY_OK;
}

int emmy_shard_range(emmy_module_t m, int ndev, int d, uint64_t *begin, uint64_t *end) {
    if (!m || ndev <= 0 || d < 0 || d >= ndev || !begin || !end)
        return fail(EMMY_ERR_INVALID, "emmy_shard_range: bad argument");
    if (!has_range(m)) return fail(EMMY_ERR_INVALID, "module takes no unit range (launch record has no EMMY_LR_RANGE)");
    const uint64_t total = m->rec.range_total, al = m->rec.range_align ? m->rec.range_align : 1;
    const uint64_t units = (total + al - 1) / al;  // aligned blocks, spread as evenly as possible
    const uint64_t lo = units * static_cast<uint64_t>(d) / static_cast<uint64_t>(ndev);
    const uint64_t hi = units * static_cast<uint64_t>(d + 1) / static_cast<uint64_t>(ndev);
    *begin = std::min(total, lo * al);
    *end = std::min(total, hi * al);
    return EMMY_OK;
}

int emmy_launch_sharded(const emmy_module_t *mods, int ndev, const uint64_t *const *args, int nargs,
                        const uint64_t *streams) {
    if (!mods || ndev <= 0 || !args) return fail(EMMY_ERR_INVALID, "emmy_launch_sharded: NULL argument");
    if (nargs < 0 || nargs > EMMY_LR_MAX_PARAMS)
        return fail(EMMY_ERR_INVALID, "emmy_launch_sharded: %d parameters (at most %d)", nargs, EMMY_LR_MAX_PARAMS);
    std::lock_guard<std::mutex> lk(g_mu);
    for (int d = 0; d < ndev; ++d) {
        emmy_module *m = mods[d];
        if (!m || (nargs > 0 && !args[d])) return fail(EMMY_ERR_INVALID, "emmy_launch_sharded: NULL module or args");
        if (!has_range(m))
            return fail(EMMY_ERR_INVALID, "module takes no unit range (launch record has no EMMY_LR_RANGE)");
        if (m->rec.range_total != mods[0]->rec.range_total || m->rec.nparams != mods[0]->rec.nparams)
            return fail(EMMY_ERR_INVALID, "emmy_launch_sharded: modules of different kernels");
    }
    for (int d = 0; d < ndev; ++d) {
        emmy_module *m = mods[d];
        const uint64_t total = m->rec.range_total, al = m->rec.range_align ? m->rec.range_align : 1;
        const uint64_t units = (total + al - 1) / al;
        const uint64_t b = std::min(total, units * d / ndev * al), e = std::min(total, units * (d + 1) / ndev * al);
        if (b == e) continue;
        // a streamed parameter holds only this device's units: rebase it so that
        // unit u sits at base + u * bytes_per_unit (modular 64-bit arithmetic)
        std::vector<uint64_t> w(args[d], args[d] + nargs);
        for (int i = 0; i < nargs && i < EMMY_LR_MAX_PARAMS; ++i)
            if (m->rec.range_bytes[i] && m->rec.param_kind[i] == EMMY_PARAM_PTR) w[i] -= b * m->rec.range_bytes[i];
        int rc = launch_locked(m, w.data(), nargs, nullptr, nullptr, streams ? streams[d] : 0, b, e);
        if (rc) return rc;
    }
    return EMMY_OK;
}

int emmy_module_range(emmy_module_t m, uint64_t *total, uint32_t *align, uint64_t *bytes_per_unit, int nargs) {
    if (!m) return fail(EMMY_ERR_INVALID, "module is NULL");
    const bool r = has_range(m);
    if (total) *total = r ? m->rec.range_total : 0;
    if (align) *align = r ? (m->rec.range_align ? m->rec.range_align : 1) : 0;
    for (int i = 0; bytes_per_unit && i < nargs && i < EMMY_LR_MAX_PARAMS; ++i)
        bytes_per_unit[i] = r ? m->rec.range_bytes[i] : 0;
    return EMMY_OK;
}

int emmy_time_launch(emmy_module_t m, const uint64_t *args, int nargs, int iters, uint64_t stream,
                     float *ms_total) {
    if (!m || !ms_total || iters <= 0) return fail(EMMY_ERR_INVALID, "emmy_time_launch: bad argument");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(m->dev);
    if (rc) return rc;
    // both events are destroyed on every path, including a failed launch
    struct Events {
        CUevent e[2] = {nullptr, nullptr};
        ~Events() {
            for (CUevent ev : e)
                if (ev) g_drv.cuEventDestroy(ev);
        }
    } ev;
    CU(g_drv.cuEventCreate(&ev.e[0], CU_EVENT_DEFAULT), "cuEventCreate");
    CU(g_drv.cuEventCreate(&ev.e[1], CU_EVENT_DEFAULT), "cuEventCreate");
    CUstream s = reinterpret_cast<CUstream>(stream);
    CU(g_drv.cuEventRecord(ev.e[0], s), "cuEventRecord");
    for (int i = 0; i < iters && rc == EMMY_OK; ++i) rc = launch_locked(m, args, nargs, nullptr, nullptr, stream);
    CU(g_drv.cuEventRecord(ev.e[1], s), "cuEventRecord");
    CU(g_drv.cuEventSynchronize(ev.e[1]), "cuEventSynchronize");
    if (rc) return rc;  // a launch failed: its error, not a time
    CU(g_drv.cuEventElapsedTime(ms_total, ev.e[0], ev.e[1]), "cuEventElapsedTime");
    return EMMY_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ graphs

struct emmy_graph {
    int dev = 0;
    CUgraphExec exec = nullptr;
};

namespace {

int graph_driver() {
    if (!g_drv.cuStreamBeginCapture || !g_drv.cuStreamEndCapture || !g_drv.cuGraphInstantiateWithFlags ||
        !g_drv.cuGraphLaunch || !g_drv.cuGraphExecDestroy || !g_drv.cuGraphDestroy)
        return fail(EMMY_ERR_NO_DRIVER, "driver lacks the stream-capture / graph entry points");
    return EMMY_OK;
}

}  // namespace

extern "C" {

int emmy_graph_begin(int dev, uint64_t stream) {
    if (stream == 0) return fail(EMMY_ERR_INVALID, "emmy_graph_begin: the legacy default stream cannot be recorded");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc || (rc = graph_driver())) return rc;
    // relaxed: other threads may keep using the driver while this stream records
    CU(g_drv.cuStreamBeginCapture(reinterpret_cast<CUstream>(stream), CU_STREAM_CAPTURE_MODE_RELAXED),
       "cuStreamBeginCapture");
    return EMMY_OK;
}

int emmy_graph_end(int dev, uint64_t stream, emmy_graph_t *out) {
    if (!out) return fail(EMMY_ERR_INVALID, "emmy_graph_end: out is NULL");
    *out = nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(dev);
    if (rc || (rc = graph_driver())) return rc;
    CUgraph graph = nullptr;
    CU(g_drv.cuStreamEndCapture(reinterpret_cast<CUstream>(stream), &graph), "cuStreamEndCapture");
    CUgraphExec exec = nullptr;
    CUresult r = g_drv.cuGraphInstantiateWithFlags(&exec, graph, 0);
    g_drv.cuGraphDestroy(graph);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuGraphInstantiateWithFlags");
    auto *g = new emmy_graph;
    g->dev = dev;
    g->exec = exec;
    *out = g;
    return EMMY_OK;
}

int emmy_graph_launch(emmy_graph_t g, uint64_t stream) {
    if (!g || !g->exec) return fail(EMMY_ERR_INVALID, "emmy_graph_launch: no graph");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(g->dev);
    if (rc) return rc;
    CU(g_drv.cuGraphLaunch(g->exec, reinterpret_cast<CUstream>(stream)), "cuGraphLaunch");
    return EMMY_OK;
}

int emmy_graph_destroy(emmy_graph_t g) {
    if (!g) return EMMY_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(g->dev);
    if (rc == EMMY_OK && g->exec) g_drv.cuGraphExecDestroy(g->exec);
    delete g;
    return rc;
}

}  // extern "C"

// ------------------------------------------------------------------ NCCL

namespace {

struct Nccl {
    void *lib = nullptr;
    bool ok = false;
    decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&::ncclCommInitRankConfig) CommInitRankConfig = nullptr;
    decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&::ncclCommDestroy) CommDestroy = nullptr;
    decltype(&::ncclCommAbort) CommAbort = nullptr;
    decltype(&::ncclAllReduce) AllReduce = nullptr;
    decltype(&::ncclAllGather) AllGather = nullptr;
    decltype(&::ncclGetErrorString) GetErrorString = nullptr;
};
Nccl g_nccl;

int load_nccl() {
    if (g_nccl.ok) return EMMY_OK;
    if (!g_nccl.lib) g_nccl.lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!g_nccl.lib) return fail(EMMY_ERR_NCCL, "cannot open libnccl.so.2: %s", dlerror());
#define EMMY_NC(field, sym)                                                                 \
    g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(g_nccl.lib, sym));        \
    if (!g_nccl.field) return fail(EMMY_ERR_NCCL, "libnccl.so.2 lacks %s", sym);
    EMMY_NC(GetUniqueId, "ncclGetUniqueId")
    EMMY_NC(CommInitRankConfig, "ncclCommInitRankConfig")
    EMMY_NC(CommGetAsyncError, "ncclCommGetAsyncError")
    EMMY_NC(CommDestroy, "ncclCommDestroy")
    EMMY_NC(CommAbort, "ncclCommAbort")
    EMMY_NC(AllReduce, "ncclAllReduce")
    EMMY_NC(AllGather, "ncclAllGather")
    EMMY_NC(GetErrorString, "ncclGetErrorString")
#undef EMMY_NC
    g_nccl.ok = true;
    return EMMY_OK;
}

}  // namespace

struct emmy_comm {
    int dev = 0;
    ncclComm_t comm = nullptr;
};

namespace {

// Poll a nonblocking communicator until its pending operation settles.
int nccl_wait(emmy_comm *c, int timeout_ms, const char *what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = g_nccl.CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) return fail(EMMY_ERR_NCCL, "%s: ncclCommGetAsyncError: %s", what, g_nccl.GetErrorString(r));
        if (st == ncclSuccess) return EMMY_OK;
        if (st != ncclInProgress) return fail(EMMY_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString(st));
        if (timeout_ms > 0) {
            const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                std::chrono::steady_clock::now() - t0);
            if (el.count() > timeout_ms) {
                g_nccl.CommAbort(c->comm);
                c->comm = nullptr;
                return fail(EMMY_ERR_TIMEOUT, "%s: no progress after %d ms; communicator aborted", what, timeout_ms);
            }
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int stream_wait(emmy_comm *c, uint64_t stream, int timeout_ms, const char *what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        CUresult r = g_drv.cuStreamQuery(reinterpret_cast<CUstream>(stream));
        if (r == CUDA_SUCCESS) return EMMY_OK;
        if (r != CUDA_ERROR_NOT_READY) return cu_fail(r, what);
        int rc = EMMY_OK;
        ncclResult_t st = ncclSuccess;
        if (g_nccl.CommGetAsyncError(c->comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress)
            rc = fail(EMMY_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString(st));
        if (!rc && timeout_ms > 0) {
            const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                std::chrono::steady_clock::now() - t0);
            if (el.count() > timeout_ms)
                rc = fail(EMMY_ERR_TIMEOUT, "%s: collective not complete after %d ms; communicator aborted",
                          what, timeout_ms);
        }
        if (rc) {
            g_nccl.CommAbort(c->comm);
            c->comm = nullptr;
            return rc;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(10));
    }
}

}  // namespace

extern "C" {

int emmy_comm_unique_id(uint8_t id[128]) {
    if (!id) return fail(EMMY_ERR_INVALID, "id is NULL");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId uid;
    ncclResult_t r = g_nccl.GetUniqueId(&uid);
    if (r != ncclSuccess) return fail(EMMY_ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.GetErrorString(r));
    static_assert(sizeof(uid) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(id, &uid, 128);
    return EMMY_OK;
}

int emmy_comm_init(int dev, int nranks, int rank, const uint8_t id[128], int timeout_ms, emmy_comm_t *out) {
    if (!id || !out || nranks <= 0 || rank < 0 || rank >= nranks)
        return fail(EMMY_ERR_INVALID, "emmy_comm_init: bad argument");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = load_nccl();
    if (rc) return rc;
    if ((rc = set_device(dev))) return rc;
    ncclUniqueId uid;
    std::memcpy(&uid, id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    auto *c = new emmy_comm();
    c->dev = dev;
    ncclResult_t r = g_nccl.CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return fail(EMMY_ERR_NCCL, "ncclCommInitRankConfig: %s", g_nccl.GetErrorString(r));
    }
    if ((rc = nccl_wait(c, timeout_ms, "ncclCommInitRankConfig"))) {
        delete c;
        return rc;
    }
    *out = c;
    return EMMY_OK;
}

int emmy_allreduce_f32(emmy_comm_t c, uint64_t send, uint64_t recv, size_t count, uint64_t stream,
                       int timeout_ms) {
    if (!c || !c->comm) return fail(EMMY_ERR_INVALID, "communicator is not live");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(c->dev);
    if (rc) return rc;
    ncclResult_t r = g_nccl.AllReduce(reinterpret_cast<const void *>(send), reinterpret_cast<void *>(recv),
                                      count, ncclFloat32, ncclSum, c->comm,
                                      reinterpret_cast<cudaStream_t>(stream));
    if (r != ncclSuccess && r != ncclInProgress)
        return fail(EMMY_ERR_NCCL, "ncclAllReduce: %s", g_nccl.GetErrorString(r));
    if ((rc = nccl_wait(c, timeout_ms, "ncclAllReduce"))) return rc;
    return stream_wait(c, stream, timeout_ms, "ncclAllReduce");
}

int emmy_allgather_f32(emmy_comm_t c, uint64_t send, uint64_t recv, size_t count_per_rank,
                       uint64_t stream, int timeout_ms) {
    if (!c || !c->comm) return fail(EMMY_ERR_INVALID, "communicator is not live");
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = set_device(c->dev);
    if (rc) return rc;
    ncclResult_t r = g_nccl.AllGather(reinterpret_cast<const void *>(send), reinterpret_cast<void *>(recv),
                                      count_per_rank, ncclFloat32, c->comm,
                                      reinterpret_cast<cudaStream_t>(stream));
    if (r != ncclSuccess && r != ncclInProgress)
        return fail(EMMY_ERR_NCCL, "ncclAllGather: %s", g_nccl.GetErrorString(r));
    if ((rc = nccl_wait(c, timeout_ms, "ncclAllGather"))) return rc;
    return stream_wait(c, stream, timeout_ms, "ncclAllGather");
}

int emmy_comm_destroy(emmy_comm_t c) {
    if (!c) return EMMY_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = EMMY_OK;
    if (c->comm) {
        set_device(c->dev);
        ncclResult_t r = g_nccl.CommDestroy(c->comm);
        if (r != ncclSuccess) rc = fail(EMMY_ERR_NCCL, "ncclCommDestroy: %s", g_nccl.GetErrorString(r));
    }
    delete c;
    return rc;
}

int emmy_comm_abort(emmy_comm_t c) {
    if (!c) return EMMY_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    if (c->comm) g_nccl.CommAbort(c->comm);
    delete c;
    return EMMY_OK;
}

}  // extern "C"
