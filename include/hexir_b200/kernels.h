/*
 * hexir_b200/kernels.h -- kernel-level C ABI of the sm_100a hot path.
 *
 * These are the GPU counterparts of the reference runtime's CPU kernels
 * (runtime/src/kernels/reference_kernels.h:17-19):
 *
 *   hexir_ref_matmul_f64(a, b, c, m, n, k)   -> hexir_cuda_matmul_f64
 *   hexir_ref_add_f64(a, b, c, n)            -> hexir_cuda_add_f64
 *   hexir_ref_relu_f64(x, y, n)              -> hexir_cuda_relu_f64
 *
 * with the same argument order and meaning, plus the CUDA ordinal the device
 * pointers belong to, a CUstream (NULL = the legacy default stream) and, for
 * matmul, flags.  Pointers are device addresses (from hexir_buffer_device_pointer,
 * cuMemAlloc, or any allocator using the device's primary context, e.g.
 * PyTorch).  Calls are asynchronous; hexir_cuda_synchronize waits and reports
 * kernel-side errors.
 *
 * Results: add and relu are bit-for-bit the reference's.  matmul sums each
 * output in a different order than the reference's sequential k loop, so it
 * agrees to f64 rounding (max |err| / max |c| <= 1e-12 in this project's
 * tests), not bit for bit.
 *
 * There is no CPU fallback: without a CUDA driver and an sm_100 GPU every call
 * returns HEXIR_ERROR_DEVICE with a message in hexir_cuda_last_error().
 */
#ifndef HEXIR_B200_KERNELS_H
#define HEXIR_B200_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#include "hexir_runtime/status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* matmul flags */
#define HEXIR_MATMUL_RELU 0x1u          /* c = relu(a . b), reference relu */
#define HEXIR_MATMUL_FORCE_TMA 0x100u   /* tests: only the TMA kernel */
#define HEXIR_MATMUL_FORCE_GUARDED 0x200u /* tests: only the guarded kernel */
/* c is another GPU's memory (a peer or IPC mapping): the kernels fence their
 * stores at system scope before finishing. */
#define HEXIR_MATMUL_REMOTE_OUTPUT 0x400u
/* Stream-K schedule for 128-row tiles (the k units of the last waves' tiles
 * dealt out evenly over one CTA per SM, split tiles summed by a fix-up
 * kernel in CTA order).  The planner takes it by itself where its wave
 * model would split k (too few tiles to fill the GPU's waves), and on
 * FORCE_STREAM_K elsewhere; never where a k split is requested or c_in is
 * given.  NO_STREAM_K rules it out: a caller that computes a matmul's rows
 * in separate calls passes it, because stream-K's sums depend on the whole
 * tile set, so row pieces would not have the bits of one call. */
#define HEXIR_MATMUL_NO_STREAM_K 0x800u
#define HEXIR_MATMUL_FORCE_STREAM_K 0x2000u
/* tests: split the k range into S pieces (1..255; any S rules out stream-K);
 * 0 = choose automatically */
#define HEXIR_MATMUL_SPLIT_K(S) (((uint32_t)(S) & 0xFFu) << 16)

/* c[m x n] = a[m x k] . b[k x n] (row-major f64), optionally relu'd.
 * Replaces hexir_ref_matmul_f64 (runtime/src/kernels/reference_kernels.c:3).
 * k == 0 gives zeros.  May use a per-device split-K workspace that the
 * library allocates once and grows on demand. */
hexir_status_t hexir_cuda_matmul_f64(int ordinal, const double *a,
                                     const double *b, double *c, uint32_t m,
                                     uint32_t n, uint32_t k, uint32_t flags,
                                     void *stream);

/* c = epilogue(c_in + a . b), with a's rows `lda` elements apart (lda >= k,
 * 0 = k) and c_in NULL (sums start at 0), equal to c, or another [m x n]
 * buffer.  Extension, no reference counterpart: it lets a product be
 * computed over consecutive k ranges -- a + k0 with lda = K, b + k0 * n,
 * each call continuing from the previous one's c -- while the next range of
 * the operands is still being copied or broadcast.  This call never splits
 * its k range (HEXIR_MATMUL_SPLIT_K(S) with S > 1 is refused), so the pieces
 * perform exactly the operations of one hexir_cuda_matmul_f64 call over all
 * of K whose plan neither splits k nor is stream-K (k0 a multiple of 32;
 * hexir_cuda_matmul_plan reports the plan), and the result has
 * the same bits; HEXIR_MATMUL_RELU belongs on the last piece only. */
hexir_status_t hexir_cuda_matmul_acc_f64(int ordinal, const double *a,
                                         uint32_t lda, const double *b,
                                         const double *c_in, double *c,
                                         uint32_t m, uint32_t n, uint32_t k,
                                         uint32_t flags, void *stream);

/* c = epilogue(a . b + addend), addend [m x n] like c: a linear and the add
 * that is its only user as one kernel (HEXIR_MATMUL_RELU applies the relu
 * after the add).  Replaces hexir_ref_matmul_f64 followed by
 * hexir_ref_add_f64 (runtime/src/kernels/reference_kernels.c:3,15): the
 * product is rounded to f64 before the add, so the result has the bits of
 * hexir_cuda_matmul_f64 then hexir_cuda_add_f64 under the same k split.
 * addend may equal c. */
hexir_status_t hexir_cuda_matmul_add_f64(int ordinal, const double *a,
                                         const double *b, const double *addend,
                                         double *c, uint32_t m, uint32_t n,
                                         uint32_t k, uint32_t flags,
                                         void *stream);

/* c[i] = a[i] + b[i] for i < n.  Replaces hexir_ref_add_f64
 * (runtime/src/kernels/reference_kernels.c:15). */
hexir_status_t hexir_cuda_add_f64(int ordinal, const double *a,
                                  const double *b, double *c, size_t n,
                                  void *stream);

/* y[i] = x[i] > 0 ? x[i] : 0 for i < n.  Replaces hexir_ref_relu_f64
 * (runtime/src/kernels/reference_kernels.c:20). */
hexir_status_t hexir_cuda_relu_f64(int ordinal, const double *x, double *y,
                                   size_t n, void *stream);

/* Activation codes: the kernel kind numbers of hexir_runtime/program.h. */
#define HEXIR_ACTIVATION_LEAKY_RELU 7u /* x > 0 ? x : 0.01 x */
#define HEXIR_ACTIVATION_ELU 8u        /* x > 0 ? x : expm1(x) (alpha 1) */
#define HEXIR_ACTIVATION_SIGMOID 9u    /* 1 / (1 + exp(-x)) */
#define HEXIR_ACTIVATION_TANH 10u      /* tanh(x) */
#define HEXIR_ACTIVATION_SOFTMAX 11u   /* exp(x - max) / sum, along each row */
#define HEXIR_ACTIVATION_GELU 12u      /* 0.5 x erfc(-x / sqrt 2) */
#define HEXIR_ACTIVATION_SWISH 13u     /* x / (1 + exp(-x)) */
#define HEXIR_ACTIVATION_MISH 14u      /* x tanh(softplus(x)) */

/* y = op(x) for a row-major [rows x cols] f64 tensor: softmax along each
 * row, every other op elementwise over rows * cols.  No reference kernel
 * exists: the reference declares these ops
 * (include/hexir/Dialect/Hexir/IR/HexirOps.td:189-308) without lowering
 * them.  The formulas above are its op descriptions; results agree with the
 * host backend's (C library functions) to a few units in the last place,
 * softmax to its row sum's rounding.  x and y may be the same buffer. */
hexir_status_t hexir_cuda_activation_f64(int ordinal, uint32_t op,
                                         const double *x, double *y,
                                         uint64_t rows, uint32_t cols,
                                         void *stream);

/* Wait for `stream` and report any error a kernel of this library recorded
 * on the device since the last check (the error word is then cleared). */
hexir_status_t hexir_cuda_synchronize(int ordinal, void *stream);

/* Which matmul kernel a call with these arguments would launch:
 * 1 = TMA pipeline with 128-row tiles, 2 = guarded (any shape/alignment),
 * 3 = TMA with 16-row tiles (m <= 16), 4 = TMA with 64-row tiles
 * (16 < m <= 64), 5 = the 128-row pipeline as a stream-K launch; *split_k
 * receives the k split (for 5: the number of CTAs sharing the k units). */
hexir_status_t hexir_cuda_matmul_plan(int ordinal, const double *a,
                                      const double *b, double *c, uint32_t m,
                                      uint32_t n, uint32_t k, uint32_t flags,
                                      int *variant, uint32_t *split_k);

/* MEASUREMENT BASELINE, not a product path: c = a . b with the schedule the
 * reference's compiler generates for a cuda-placed hexir.linear
 * (compiler/Conversion/HexirToTIR/HexirToTIR.cpp:82-170), restated in CUDA
 * C: one thread per output, grid (n / bs, m), block bs = the largest power
 * of two <= 256 dividing n, serial k with one fused multiply-add per step,
 * operands read from global memory.  m > 65535 is refused
 * (INVALID_ARGUMENT), as the reference's grid.y cannot launch it.
 * Asynchronous on `stream`. */
hexir_status_t hexir_cuda_baseline_reference_schedule_f64(
    int ordinal, const double *a, const double *b, double *c, uint32_t m,
    uint32_t n, uint32_t k, void *stream);

/* FP64 tensor-core throughput probe: one launch of `blocks` CTAs x 256
 * threads, each warp running `iters` rounds of 8 dependent-free DMMAs.
 * *flops receives the launch's FLOP count.  `out` must hold blocks*256 f64. */
hexir_status_t hexir_cuda_dmma_probe(int ordinal, double *out, uint32_t blocks,
                                     uint32_t iters, void *stream,
                                     double *flops);

/* Failure-detection probe: a one-thread kernel waits on a barrier nothing
 * arrives at and gives up after timeout_ns, recording a wait timeout in the
 * device error word.  The next hexir_cuda_synchronize then returns
 * HEXIR_ERROR_DEVICE; the context stays usable.  Every wait in this library's
 * kernels is bounded the same way (4 s), so a stuck pipeline ends with an
 * error status instead of a hung GPU. */
hexir_status_t hexir_cuda_wait_probe(int ordinal, uint64_t timeout_ns,
                                     void *stream);

/* Size of the fixed scratch array behind hexir_cuda_matmul_f64_noalloc. */
#define HEXIR_NOALLOC_SCRATCH_BYTES (16u << 20)

/* c = a . b like hexir_cuda_matmul_f64, for callers that cannot allocate
 * device memory.  No counterpart in the reference.
 *
 * Who needs it: code that runs where allocating is not allowed or not
 * affordable -- an application whose device memory is fully owned by its own
 * pool allocator, a latency-bound service that cannot take the device-wide
 * synchronisation cudaFree implies, a caller that budgets all device memory
 * at start-up.  hexir_cuda_matmul_f64 may allocate (and grow) a split-K
 * workspace; this entry point never calls cudaMalloc, cudaFree or any other
 * allocating routine.  Its split-K partial sums go to a fixed
 * HEXIR_NOALLOC_SCRATCH_BYTES array of device memory that comes with the
 * library's device code: each GPU the library's device code is loaded on
 * holds it until the process exits.
 *
 * The caller still provides a, b and c.  Shapes whose partial sums do not fit
 * the array (split * m * n * 8 bytes) are rejected with
 * HEXIR_ERROR_INVALID_ARGUMENT and a message in hexir_cuda_last_error().
 * The kernel is the bounds-checked DMMA GEMM (any shape and alignment), so
 * results agree with hexir_cuda_matmul_f64 to f64 rounding, not bit for bit.
 *
 * The first call on a device sets that device up (looks up the array's device
 * address with the device current); make it before any stream capture.
 * Every call on a device shares the one array, which keeps the last call's
 * contents; nothing in it needs to start at zero, but calls whose kernels
 * overlap on the GPU race on it and must be serialised by the caller. */
hexir_status_t hexir_cuda_matmul_f64_noalloc(int ordinal, const double *a,
                                             const double *b, double *c,
                                             uint32_t m, uint32_t n, uint32_t k,
                                             uint32_t flags, void *stream);

/* Kernel launches issued by this library since the process started. */
uint64_t hexir_cuda_launch_count(void);

/* Multiprocessor count of a device (0 if unavailable). */
int hexir_cuda_sm_count(int ordinal);

/* The sm_100a kernel image this library launches (a CUBIN built from
 * hexir_b200/csrc/kernels/kernels.cu), as embedded in the library. */
hexir_status_t hexir_cuda_kernel_image(const void **data, size_t *size);

/* Message of the last failed call on this thread ("" if none). */
const char *hexir_cuda_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_B200_KERNELS_H */
