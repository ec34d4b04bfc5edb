/*
 * launch_abi.h -- by-value argument blocks of the sm_100a kernels.
 *
 * Shared by the device code (the .cu files under kernels/) and the host launcher
 * (runtime/kernel_lib.cc), which passes each block by value through
 * cuLaunchKernel.  Plain C, fixed-width fields, no pointers to host memory.
 */
#ifndef HEXIR_B200_LAUNCH_ABI_H
#define HEXIR_B200_LAUNCH_ABI_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Tile shape of the TMA-fed DMMA GEMM (linear_f64.cu). */
#define HEXIR_LINEAR_BM 128
#define HEXIR_LINEAR_BN 128
#define HEXIR_LINEAR_BK 32
#define HEXIR_LINEAR_STAGES 3
#define HEXIR_LINEAR_CONSUMER_WARPS 8
#define HEXIR_LINEAR_THREADS (HEXIR_LINEAR_CONSUMER_WARPS * 32)
/* A stage: BK/8 slabs of [BM][8] f64; B stage: BN/16 slabs of [BK][16] f64. */
#define HEXIR_LINEAR_STAGE_BYTES \
  ((HEXIR_LINEAR_BM * HEXIR_LINEAR_BK + HEXIR_LINEAR_BK * HEXIR_LINEAR_BN) * 8)
/* + 1024 for aligning the ring to the 128-byte swizzle atom, + barriers. */
#define HEXIR_LINEAR_SMEM_BYTES \
  (HEXIR_LINEAR_STAGES * HEXIR_LINEAR_STAGE_BYTES + 1024 + 256)

/* Shared memory of the 64-row (4 stages) and 16-row (3 stages, two CTAs per
 * SM) variants. */
#define HEXIR_LINEAR_M64_SMEM_BYTES \
  (4 * ((64 * 32 + 32 * 128) * 8) + 1024 + 256)
#define HEXIR_LINEAR_M16_SMEM_BYTES \
  (3 * ((16 * 32 + 32 * 128) * 8) + 1024 + 256)

/* Tile shape of the guarded GEMM for shapes TMA cannot describe. */
#define HEXIR_LINEAR_G_BM 64
#define HEXIR_LINEAR_G_BN 64
#define HEXIR_LINEAR_G_BK 16
#define HEXIR_LINEAR_G_THREADS 128
#define HEXIR_LINEAR_G_SMEM_BYTES \
  (2 * (HEXIR_LINEAR_G_BM * HEXIR_LINEAR_G_BK + \
        HEXIR_LINEAR_G_BK * HEXIR_LINEAR_G_BN) * 8 + 1024)

#define HEXIR_EPILOGUE_RELU 0x1u
/* c is another GPU's memory (peer / IPC mapping): fence the stores at system
 * scope before the CTA exits, so the owner sees them once it has synchronised
 * with this kernel's completion. */
#define HEXIR_EPILOGUE_SYSTEM_FENCE 0x2u
/* c (and c_in) rows start on 32-byte boundaries (n % 4 == 0, 32-byte aligned
 * base): the TMA kernels move each thread's four consecutive outputs with one
 * 256-bit access, so a warp's store covers whole 128-byte lines. */
#define HEXIR_EPILOGUE_VEC4 0x4u
/* c = a . b + addend (then the relu, if set): a linear and the add that is
 * its only user, fused.  Same rounding as the two kernels: the sum is an f64
 * before the add. */
#define HEXIR_EPILOGUE_ADD 0x8u
/* The output is final (no split-K partial another kernel reads): store it
 * with the streaming cache hint (evict first). */
#define HEXIR_EPILOGUE_STREAM 0x10u

/* CTAs per tile of the stream-K fix-up (grid.y). */
#define HEXIR_SK_FIXUP_PARTS 16u

/* Error bits a kernel ORs into the device error word. */
#define HEXIR_KERR_WAIT_TIMEOUT 0x1u  /* a pipeline wait ran out of time */
#define HEXIR_KERR_BAD_ARGS 0x2u      /* launch arguments failed a check */

typedef struct {
  double *c;             /* destination (or split-K partials), row-major */
  const double *a;       /* [m][k] row-major; read by the guarded kernel */
  const double *b;       /* [k][n] row-major; read by the guarded kernel */
  uint32_t m, n, k;
  uint32_t epilogue;     /* HEXIR_EPILOGUE_* applied when split_k == 1 */
  uint32_t tiles_m, tiles_n;
  uint32_t group_m;      /* tile raster: group_m row-tiles per column sweep */
  uint32_t k_tiles;      /* ceil(k / BK) */
  uint32_t split_k;      /* K ranges; > 1 writes partials to c + s*m*n */
  uint32_t k_tiles_per_split;
  unsigned int *error;   /* device error word */
  uint64_t timeout_ns;   /* bound on every pipeline wait */
  /* Non-null: each element's sum starts from c_in (same [m][n] layout as c,
   * may equal c) instead of 0.0, so a product computed over consecutive k
   * ranges, each launch continuing from the last one's output, performs the
   * same operations in the same order as one launch over all of k.  Only
   * with split_k == 1. */
  const double *c_in;
  uint32_t lda;          /* row stride of a in elements (>= k) */
  uint32_t reserved;
  const double *addend;  /* [m][n], with HEXIR_EPILOGUE_ADD */
  /* Stream-K launches (hexir_linear_f64_tma_sk): tiles below sk_dp_tiles go
   * whole to CTAs c, c + G, ... (G = gridDim.x); the k-tile units of the
   * rest are dealt out in consecutive runs of sk_units per CTA.  A tile whose
   * units span CTAs leaves each CTA's partial sums in sk_partials (slot 2c
   * for the CTA's first tile of the run, 2c + 1 for its last), which
   * hexir_linear_f64_sk_fixup sums in CTA order. */
  uint32_t sk_dp_tiles;
  uint32_t sk_units;
  double *sk_partials;   /* [2 G][BM][BN] */
} hexir_linear_args_t;

typedef struct {
  const double *partials; /* [split][m*n] */
  double *c;
  uint64_t count;         /* m * n */
  uint32_t split;
  uint32_t epilogue;
  const double *addend;   /* [m*n], with HEXIR_EPILOGUE_ADD */
} hexir_reduce_args_t;

typedef struct {
  const double *x;
  const double *y; /* second operand of add; unused by relu */
  double *out;
  uint64_t count;
} hexir_elementwise_args_t;

/* Activation codes: the kernel kind numbers of program.h (7-14). */
#define HEXIR_ACT_LEAKY_RELU 7u
#define HEXIR_ACT_ELU 8u
#define HEXIR_ACT_SIGMOID 9u
#define HEXIR_ACT_TANH 10u
#define HEXIR_ACT_SOFTMAX 11u
#define HEXIR_ACT_GELU 12u
#define HEXIR_ACT_SWISH 13u
#define HEXIR_ACT_MISH 14u
/* The fixed slopes of leaky_relu and elu (the ops carry no attribute). */
#define HEXIR_LEAKY_RELU_ALPHA 0.01
#define HEXIR_ELU_ALPHA 1.0

/* Softmax launch shapes: a warp per row up to 32 x 32 columns, a 256-thread
 * block per row up to 256 x 32, a 512-thread block per row up to 512 x 32
 * (each thread holding up to 32 elements in registers), and above that a
 * 512-thread block per row that reads the row three times.  Rows of an even
 * length starting 16-byte aligned, above the warp shape, run the persistent
 * "bulk" blocks instead: the next row is copied into shared memory
 * (cp.async.bulk) while the current one computes. */
#define HEXIR_SOFTMAX_WARP_COLS 1024u
#define HEXIR_SOFTMAX_B256_COLS 8192u
#define HEXIR_SOFTMAX_B512_COLS 16384u
// Short rows through the bulk-prefetch blocks: fewer elements per thread,
// more blocks per SM (5 up to 2048 columns, 3 up to 4096).
#define HEXIR_SOFTMAX_S2K_COLS 2048u
#define HEXIR_SOFTMAX_S4K_COLS 4096u

typedef struct {
  const double *x;
  double *out;
  uint64_t count; /* elementwise: elements; softmax: rows * cols */
  uint64_t rows;  /* softmax rows */
  uint32_t cols;  /* softmax row length */
  uint32_t op;    /* HEXIR_ACT_* */
  uint64_t timeout_ns; /* bound on every wait (the bulk softmax) */
} hexir_activation_args_t;

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_B200_LAUNCH_ABI_H */
