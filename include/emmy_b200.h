/*
 * libemmy_b200 - C ABI of the emmy B200 execution backend.
 *
 * The reference (vedantgpt/emmy-ptx-compiler) stops at printing PTX; an
 * external runner (the starter kit's submit.py and a hosted GPU service,
 * reference README.md:170-182) assembled that PTX, launched the entry under
 * meta.json's grid/block/smem_bytes on device buffers, and compared the
 * outputs.  This library is that missing launch layer, for modules produced
 * by our compiler (compile_bundle, reference compile.py:3168-3215) and for
 * any other PTX/cubin module, such as the reference's own output.
 *
 * Conventions: every function returns 0 (EMMY_OK) or a negative EMMY_ERR_*
 * code and never aborts the process; emmy_last_error() gives the message of
 * the calling thread's last failure.  Device pointers and streams are plain
 * 64-bit integers (CUdeviceptr / CUstream of the device's primary context,
 * which is also the context the CUDA runtime and PyTorch use).  The caller
 * owns device buffers; the library owns modules and communicators.
 * libcuda and libnccl are opened at run time, so the library itself loads on
 * machines without a GPU driver.
 */
#ifndef EMMY_B200_H
#define EMMY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMMY_OK 0
#define EMMY_ERR_NO_DRIVER (-1)     /* libcuda.so.1 could not be opened or cuInit failed */
#define EMMY_ERR_CUDA (-2)          /* a driver call failed; see emmy_last_error */
#define EMMY_ERR_INVALID (-3)       /* bad argument */
#define EMMY_ERR_NOT_FOUND (-4)     /* entry / symbol / device not found */
#define EMMY_ERR_KERNEL_STATUS (-5) /* a kernel raised EMMY_STATUS_* bits */
#define EMMY_ERR_TIMEOUT (-6)       /* a bounded host wait ran out */
#define EMMY_ERR_NCCL (-7)          /* NCCL missing or a collective failed */
#define EMMY_ERR_NOT_INIT (-8)      /* emmy_init has not succeeded */

typedef struct emmy_module *emmy_module_t;
typedef struct emmy_comm *emmy_comm_t;

/* Library version string, e.g. "emmy_b200 1.0 (sm_100a)". */
const char *emmy_version(void);

/* Thread-local message of the last failed call; returns the code of that call. */
int emmy_last_error(char *buf, size_t len);

/* Open libcuda, cuInit, retain the primary context of devices [0, ndev)
 * (ndev <= 0: every device).  Replaces the runner's device setup. */
int emmy_init(int ndev);

int emmy_device_count(int *count);

/* Load a PTX (NUL-terminated text) or cubin image on device `dev` and resolve
 * `entry` (the reference's `.visible .entry <KernelOp.name>`,
 * compile.py:862).  Modules from our compiler also carry a launch record
 * (include/emmy_launch_record.h), read here.
 *
 * Entries of our modules: `<entry>` itself always takes exactly the meta.json
 * arg_order parameters and is correct under the reference runner's launch
 * (meta grid, block, smem_bytes).  When the fast kernel needs more - a unit
 * range after the buffers, TMA tensor maps, a thread-block cluster - the
 * module also exports it as `<entry>__emmy`, and this library launches that
 * one (with the record's geometry and extras).  Full-array reductions also
 * export `<entry>__xchg` (emmy_launch_xchg).
 *
 * Reduction modules whose blocks split a row keep their cross-block partials
 * and per-row arrival counters in globals of the loaded module (created
 * zeroed by the load; the block that completes a row resets its counter).
 * So do tensor-core attention modules launched as a cooperative grid
 * (EMMY_LR_COOPERATIVE in the record): the CTAs of a query tile exchange row
 * values and partial outputs there, behind a per-tile arrival counter that
 * every completed launch leaves at a multiple of the tile's CTA count.
 * Two launches of ONE loaded module that overlap on the GPU (two streams)
 * race on them: serialise them, or load the module once per stream.  A launch
 * that does not run to completion (its context is then lost) leaves the
 * counters undefined: unload and load the module again before reusing it. */
int emmy_load(int dev, const void *image, size_t len, const char *entry, emmy_module_t *out);

int emmy_unload(emmy_module_t m);

/* The module's launch record: family (0 when the module has none), tuned
 * grid/block, dynamic shared memory and IR parameter count. */
int emmy_module_info(emmy_module_t m, uint32_t *family, uint32_t grid[3], uint32_t block[3],
                     uint32_t *dyn_smem, uint32_t *nparams);

/* Launch the entry.  `args` holds one 64-bit word per IR parameter in
 * meta.json arg_order (compile.py:314-317, 854-864): a device pointer, or
 * the bits of an f32 / i32 scalar in the low 32 bits.  grid/block NULL
 * means the module's launch record; modules without one need both.  Tensor
 * maps the record describes are encoded and appended after the IR
 * parameters.  Asynchronous on `stream` (0 = the legacy default stream). */
int emmy_launch(emmy_module_t m, const uint64_t *args, int nargs, const uint32_t *grid,
                const uint32_t *block, uint64_t stream);

/* The reference runner's whole meta.json launch (grid, block and smem_bytes:
 * reference README.md:170-182, tools/make_proxy_set.py:75-86): emmy_launch
 * with explicit geometry and `dyn_smem` bytes of dynamic shared memory, for
 * modules that size `.extern .shared` at launch (the reference's PTX above 48
 * KiB, compile.py:827-836).  The function's dynamic shared-memory limit is
 * raised when `dyn_smem` needs it. */
int emmy_launch_ex(emmy_module_t m, const uint64_t *args, int nargs, const uint32_t *grid,
                   const uint32_t *block, uint32_t dyn_smem, uint64_t stream);

/* Read and clear the module's device status word (EMMY_STATUS_* bits from
 * include/emmy_launch_record.h).  Synchronises the device first. */
int emmy_module_status(emmy_module_t m, uint32_t *status);

/* Wait for `stream` on `dev`, polling, for at most timeout_ms (<= 0: no limit). */
int emmy_sync(int dev, uint64_t stream, int timeout_ms);

/* Device memory and copies, for hosts without another CUDA runtime. */
int emmy_alloc(int dev, size_t bytes, uint64_t *dptr);
int emmy_free(int dev, uint64_t dptr);
int emmy_memcpy_htod(int dev, uint64_t dst, const void *src, size_t bytes, uint64_t stream);
int emmy_memcpy_dtoh(int dev, void *dst, uint64_t src, size_t bytes, uint64_t stream);
int emmy_memset_d8(int dev, uint64_t dst, uint8_t value, size_t bytes, uint64_t stream);
int emmy_host_alloc(size_t bytes, void **ptr);  /* pinned host memory */
int emmy_host_free(void *ptr);

/* Argument roles of emmy_run_host. */
#define EMMY_ROLE_IN 0          /* host -> device before the launch */
#define EMMY_ROLE_OUT 1         /* device -> host after the launch */
#define EMMY_ROLE_INOUT 2       /* both */
#define EMMY_ROLE_OUT_ZEROED 3  /* zero-filled on the device, then device -> host (meta zero_outputs) */
#define EMMY_ROLE_SCALAR 4      /* host_ptrs[i] points at the 4-byte scalar value */

/* Run the entry on host buffers - the whole job the reference's runner did
 * per problem (README.md:170-182): copy inputs in, zero `zero_outputs`,
 * launch with the module's record, copy outputs back.  Device buffers are
 * owned by the module and reused across calls; everything is ordered on
 * `stream`, and the call returns after the outputs are on the host. */
int emmy_run_host(emmy_module_t m, void *const *host_ptrs, const size_t *bytes,
                  const uint8_t *roles, int nargs, uint64_t stream);

/* Launch over units [begin, end) only (no counterpart in the reference):
 * modules whose launch record carries EMMY_LR_RANGE (pointwise: cells, GEMM:
 * output rows) read and write only those units' bytes of the streamed
 * parameters, so a caller can overlap copies of one range with the kernel
 * on another.  begin and end are multiples of the module's alignment (end may
 * be the total); emmy_module_range reports total, alignment and the bytes per
 * unit of each parameter (0 = read whole).  emmy_run_host uses this to pipeline
 * large problems in chunks over a copy-in stream, `stream` and a copy-out
 * stream. */
int emmy_launch_range(emmy_module_t m, const uint64_t *args, int nargs, uint64_t begin, uint64_t end,
                      uint64_t stream);
int emmy_module_range(emmy_module_t m, uint64_t *total, uint32_t *align, uint64_t *bytes_per_unit, int nargs);

/* One launch split over `ndev` GPUs by unit range: the row / M split of the
 * boundary's sharded launch.  mods[d] is the kernel's module loaded on device d
 * (emmy_load(d, ...)); args[d] are that device's `nargs` parameter words.  A
 * streamed parameter (bytes per unit > 0) points at device d's shard, which
 * holds exactly its units [begin, end) from emmy_shard_range; every other
 * parameter is complete on each device.  Device d gets units
 * [floor(d*U/ndev), floor((d+1)*U/ndev)) of the U aligned blocks.  Launches are
 * asynchronous on streams[d] (NULL: each device's default stream). */
int emmy_shard_range(emmy_module_t m, int ndev, int d, uint64_t *begin, uint64_t *end);
int emmy_launch_sharded(const emmy_module_t *mods, int ndev, const uint64_t *const *args, int nargs,
                        const uint64_t *streams);

/* Launch `iters` times back to back on `stream` between two CUDA events and
 * return the elapsed milliseconds (device time). */
int emmy_time_launch(emmy_module_t m, const uint64_t *args, int nargs, int iters, uint64_t stream,
                     float *ms_total);

/* CUDA graphs of launches.  No counterpart in the reference, which leaves
 * launching to its caller.  emmy_graph_begin starts recording what is issued
 * on `stream` of device `dev` (a stream the caller created: the legacy default
 * stream 0 cannot be recorded); launches issued there are then recorded, not
 * run.  emmy_graph_end stops recording and instantiates the graph.
 * emmy_graph_launch replays every recorded launch, in order, with the argument
 * values of the recording, on `stream` (asynchronous); the modules recorded
 * must stay loaded while the graph exists.  emmy_graph_end always takes the
 * stream out of recording, also when the recording was invalidated (it then
 * returns the error and no graph).  emmy_run_host, emmy_sync and
 * emmy_time_launch synchronise, so they cannot be recorded. */
typedef struct emmy_graph *emmy_graph_t;
int emmy_graph_begin(int dev, uint64_t stream);
int emmy_graph_end(int dev, uint64_t stream, emmy_graph_t *out);
int emmy_graph_launch(emmy_graph_t g, uint64_t stream);
int emmy_graph_destroy(emmy_graph_t g);

/* Full-array f32 sum that allocates nothing.  No counterpart in the
 * reference.  For callers that may not call cudaMalloc (fixed memory budgets,
 * pre-sized pools, runtimes that own every allocation): the cross-block
 * scratch is one fixed __device__ array inside this library, of
 * EMMY_NOALLOC_SCRATCH_BYTES per GPU that loads the library, held until the
 * process exits.  Computes *out = sum(x[0..n)) on `stream` (asynchronous),
 * n <= EMMY_NOALLOC_MAX_ELEMENTS, else EMMY_ERR_INVALID.  All calls on a
 * device share the array: calls that overlap on the GPU race.  The first call
 * on each device resolves the array's address (cudaGetSymbolAddress); make it
 * before any stream capture.  The address is kept for the life of the
 * process: after cudaDeviceReset (or any reset of the device's primary
 * context) this entry point must not be called again on that device. */
#define EMMY_NOALLOC_MAX_CHUNKS 4096
#define EMMY_NOALLOC_SCRATCH_BYTES (EMMY_NOALLOC_MAX_CHUNKS * 4 + 256)
#define EMMY_NOALLOC_MAX_ELEMENTS (1ull << 36)
int emmy_sum_f32_noalloc(int dev, const float *x, uint64_t n, float *out, uint64_t stream);

/* The C4 step on N GPUs as ONE kernel per GPU (no counterpart in the
 * reference, which has no multi-GPU path): the full-array sum of this GPU's
 * shard fused with the cross-GPU combine over NVLink peer memory.
 *
 *   emmy_xchg_create   allocates this GPU's exchange buffer and returns its
 *                      CUDA IPC handle (EMMY_XCHG_HANDLE_BYTES);
 *   emmy_xchg_connect  maps every rank's buffer, given all ranks' handles in
 *                      rank order (exchanged by the caller, e.g. through
 *                      torch.distributed);
 *   emmy_sum_f32_allreduce  *out = sum over ranks of sum(data[0..n)), the same
 *                      bits on every rank (partials added in rank order).
 *                      Asynchronous on `stream`; every rank must make the same
 *                      sequence of calls (of this and of emmy_launch_xchg).
 *                      A rank whose peers do not arrive within timeout_ms
 *                      (<= 0: 1000) writes NaN and sets bit 0 of the status
 *                      word, and the group is then FAILED on that rank: every
 *                      later call returns NaN at once, without publishing,
 *                      until emmy_xchg_reset;
 *   emmy_launch_xchg   the same combine at the end of a compiled full-array
 *                      reduction KernelOp: launches the module's
 *                      <entry>__xchg kernel (this GPU's shard reduced, the
 *                      per-GPU results exchanged and combined with the
 *                      reduction's operator in rank order, the epilogue run
 *                      on the combined value), same rules as above;
 *   emmy_xchg_status   reads and clears the status word;
 *   emmy_xchg_reset    clears the buffer (and the FAILED state) and restarts
 *                      the call count: every rank must reset, with no call of
 *                      the group in flight on any rank (e.g. after a barrier
 *                      that follows a stream synchronisation);
 *   emmy_xchg_destroy  requires every peer to have stopped calling (peers
 *                      store into this GPU's buffer through their mapping).
 * At most EMMY_XCHG_MAX_RANKS ranks, one GPU each. */
#define EMMY_XCHG_MAX_RANKS 8
#define EMMY_XCHG_HANDLE_BYTES 64
typedef struct emmy_xchg *emmy_xchg_t;
int emmy_xchg_create(int dev, int nranks, int rank, emmy_xchg_t *out, uint8_t handle[EMMY_XCHG_HANDLE_BYTES]);
int emmy_xchg_connect(emmy_xchg_t x, const uint8_t *handles);
int emmy_sum_f32_allreduce(emmy_xchg_t x, const float *data, uint64_t n, float *out, int timeout_ms,
                           uint64_t stream);
int emmy_launch_xchg(emmy_module_t m, const uint64_t *args, int nargs, emmy_xchg_t x, int timeout_ms,
                     uint64_t stream);
int emmy_xchg_status(emmy_xchg_t x, uint32_t *status);
int emmy_xchg_reset(emmy_xchg_t x);
int emmy_xchg_destroy(emmy_xchg_t x);

/* NCCL over NVLink/NVSwitch for the one collective of the path: combining
 * per-GPU partials of a full-array reduction.  No reference counterpart
 * (the reference is single-GPU). */
int emmy_comm_unique_id(uint8_t id[128]);
int emmy_comm_init(int dev, int nranks, int rank, const uint8_t id[128], int timeout_ms,
                   emmy_comm_t *out);
int emmy_allreduce_f32(emmy_comm_t c, uint64_t send, uint64_t recv, size_t count, uint64_t stream,
                       int timeout_ms);
int emmy_allgather_f32(emmy_comm_t c, uint64_t send, uint64_t recv, size_t count_per_rank,
                       uint64_t stream, int timeout_ms);
int emmy_comm_destroy(emmy_comm_t c);
int emmy_comm_abort(emmy_comm_t c);

#ifdef __cplusplus
}
#endif

#endif
