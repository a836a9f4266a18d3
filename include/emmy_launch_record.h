/*
 * Launch record and status word embedded in every module the emmy B200
 * compiler emits.
 *
 * The reference compiler's modules carry no launch information: the external
 * runner launched them with meta.json's grid/block/smem_bytes (the contract
 * in the reference README, "Correct under the launch in meta.json").  Our
 * kernels are correct under any 1-D launch, but they are fastest under the
 * geometry the lowering chose, and the GEMM family needs TMA tensor maps
 * encoded on the host.  So each module exports:
 *
 *   extern "C" __device__ const EmmyLaunchRecord emmy_launch_record;
 *   extern "C" __device__ unsigned int emmy_status;
 *
 * libemmy_b200 (emmy_load) reads the record with cuModuleGetGlobal, and
 * emmy_launch appends the tensor maps it describes after the arg_order
 * parameters - the same "arg_order, then tensor-map params" layout the
 * reference uses for its own TMA descriptors (compile.py:854-864).
 * Kernels report failures (a bounded wait that ran out, a launch geometry
 * they cannot run under) by OR-ing EMMY_STATUS_* bits into emmy_status;
 * emmy_module_status() reads and clears it.
 *
 * This header is shared by device code (generated .cu files) and host code
 * (emmy_runtime.cpp), so the layout is plain fixed-width integers.
 */
#ifndef EMMY_LAUNCH_RECORD_H
#define EMMY_LAUNCH_RECORD_H

#include <stdint.h>

#define EMMY_LR_MAGIC 0x31594D45u /* "EMY1" little-endian */
#define EMMY_LR_VERSION 2u
#define EMMY_LR_MAX_PARAMS 32
#define EMMY_LR_MAX_TMAPS 4

enum EmmyFamily {
    EMMY_FAMILY_POINTWISE = 1,
    EMMY_FAMILY_REDUCTION = 2,
    EMMY_FAMILY_GEMM = 3,
    EMMY_FAMILY_ROWFUSED = 4, /* row reductions + pointwise pass in one kernel */
    EMMY_FAMILY_ATTENTION = 5, /* per-key passes over q.k scores, weighted sum of v */
    EMMY_FAMILY_SCHEDULE = 6   /* any other KernelOp, in the schedule its IR spells out */
};

enum EmmyParamKind { EMMY_PARAM_PTR = 0, EMMY_PARAM_F32 = 1, EMMY_PARAM_I32 = 2 };

/* Status bits a kernel may raise (never a trap or a fault). */
#define EMMY_STATUS_TIMEOUT_PRODUCER 0x1u /* TMA producer gave up waiting for a free stage */
#define EMMY_STATUS_TIMEOUT_MMA 0x2u      /* MMA issuer gave up waiting for data/accumulator */
#define EMMY_STATUS_TIMEOUT_EPILOGUE 0x4u /* epilogue gave up waiting for an accumulator */
#define EMMY_STATUS_BAD_LAUNCH 0x8u       /* block shape or smem the kernel cannot run under */
#define EMMY_STATUS_TMEM_ALLOC 0x10u      /* tensor-memory allocation did not fit */
#define EMMY_STATUS_TIMEOUT_REDUCE 0x20u  /* cross-block combine waited too long */

/* flags: bits 0-7 cluster size (0/1 = no cluster); EMMY_LR_FILL_GRID asks the
 * loader to size grid[0] from the kernel's occupancy on the device it is
 * loaded on: grid[0] = waves x resident CTAs per SM x SM count, rounded down
 * to a multiple of grid_quantum.  In the record as emitted, grid[0] holds the
 * number of waves; emmy_module_info reports the resolved grid. */
#define EMMY_LR_FILL_GRID 0x100u
/* EMMY_LR_RANGE: the kernel takes two more parameters after the tensor maps,
 * uint64 range_begin and range_end, and does the work of units
 * [range_begin, range_end) only (pointwise: cells; GEMM: rows of the output).
 * A launch over the whole problem passes 0 and range_total.  Unit u of a
 * parameter with range_bytes[i] > 0 is bytes [u * range_bytes[i],
 * (u + 1) * range_bytes[i]) of that buffer, and a launch over a range reads
 * and writes no other bytes of it; parameters with range_bytes[i] == 0 are
 * read whole by every launch.  Range ends are multiples of range_align, or
 * range_total.  A tensor map over a parameter with range_bytes[i] > 0 is
 * encoded per launch: it starts at the launch's first unit and its outer
 * extent is the launch's unit count (the kernel addresses it relative to
 * range_begin). */
#define EMMY_LR_RANGE 0x200u
/* EMMY_LR_GRID_UNITS (with EMMY_LR_RANGE): one CTA per grid_quantum units
 * (0 = 1) of the launch's range, at most grid[0] CTAs (the kernel strides
 * over any units beyond its grid).  A launch that passes its own grid keeps
 * it. */
#define EMMY_LR_GRID_UNITS 0x400u
/* EMMY_LR_COOPERATIVE: launched as a cooperative grid (every CTA resident at
 * once, or the launch fails): the kernel's CTAs wait on one another through
 * global memory. */
#define EMMY_LR_COOPERATIVE 0x800u

typedef struct EmmyTmapSpec {
    uint32_t src_param; /* index into arg_order of the global buffer */
    uint32_t dtype;     /* CUtensorMapDataType */
    uint32_t rank;
    uint32_t swizzle;   /* CUtensorMapSwizzle */
    uint64_t dims[5];   /* innermost first, elements */
    uint64_t strides[4];/* bytes, for dims 1..rank-1 */
    uint32_t box[5];
    uint32_t l2_promotion; /* CUtensorMapL2promotion */
    uint32_t reserved[3];
} EmmyTmapSpec;

typedef struct EmmyLaunchRecord {
    uint32_t magic;
    uint32_t version;
    uint32_t family;
    uint32_t flags;
    uint32_t grid[3];
    uint32_t block[3];
    uint32_t dyn_smem;
    uint32_t nparams;
    uint32_t param_kind[EMMY_LR_MAX_PARAMS];
    uint32_t ntmaps;
    uint32_t grid_quantum; /* EMMY_LR_FILL_GRID: grid[0] is a multiple of this; EMMY_LR_GRID_UNITS: units per CTA (0 = 1) */
    EmmyTmapSpec tmaps[EMMY_LR_MAX_TMAPS];
    /* version 2: unit ranges (EMMY_LR_RANGE) */
    uint64_t range_total;
    uint32_t range_align;
    uint32_t range_reserved;
    uint64_t range_bytes[EMMY_LR_MAX_PARAMS];
} EmmyLaunchRecord;

#endif
