/*
 * hexir_b200/comm.h -- row sharding of a linear across GPUs.
 *
 * The reference has no multi-GPU path; its placement is per op and per
 * process (compiler/Target/TargetInfo.cpp:20-45, runtime/src/vm/
 * interpreter.c:85-92).  This header adds the one strategy the hot path
 * needs: the rows of a[m x k] (and so of c[m x n]) are split over GPUs, the
 * weight b[k x n] is broadcast from the first GPU over NVLink with NCCL, every
 * GPU computes its rows with no collective, and the output rows land on the
 * first GPU.  Where the GPUs can reach the first GPU's memory (peer access in
 * one process, a CUDA IPC mapping across processes of one host), each GPU's
 * kernel stores its output tiles there directly over NVLink as it computes
 * them; otherwise the rows are gathered with NCCL send/receive.
 *
 * Two ways in:
 *   - in one process, a module whose linear is placed on "cuda:F-L" run with
 *     hexir_execute_devices (vm.h);
 *   - one process per GPU: every rank calls hexir_sharded_linear_f64 with the
 *     communicator from hexir_comm_init_rank.
 */
#ifndef HEXIR_B200_COMM_H
#define HEXIR_B200_COMM_H

#include <stddef.h>
#include <stdint.h>

#include "hexir_runtime/status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Balanced split of `rows` over `shards`: shard i gets rows
 * [*begin, *begin + *count); the first rows % shards shards get one extra. */
hexir_status_t hexir_shard_rows(uint64_t rows, uint32_t shards, uint32_t index,
                                uint64_t *begin, uint64_t *count);

/* Most pieces a rank's output rows are gathered in (the NCCL path of
 * hexir_sharded_linear_f64) and most k pieces the weight is broadcast in. */
#define HEXIR_SHARD_MAX_GATHER_PIECES 5
#define HEXIR_SHARD_MAX_WEIGHT_PIECES 2

/* Piece `index` of a rank's `rows` output rows as hexir_sharded_linear_f64
 * sends them to the root when it gathers with NCCL: rows [*begin, *begin +
 * *count) of that rank's block, *pieces the number of pieces (at most
 * HEXIR_SHARD_MAX_GATHER_PIECES; 0 for no rows).  The pieces halve in size
 * down to whole 128-row tiles of at least 256 rows, so every send but the
 * last hides behind the next piece's GEMM; an index past the last piece
 * gives *count 0.  Every rank computes every peer's pieces with this rule. */
hexir_status_t hexir_shard_gather_pieces(uint64_t rows, uint32_t index,
                                         uint64_t *begin, uint64_t *count,
                                         uint32_t *pieces);

/* The k pieces in which hexir_sharded_linear_f64 broadcasts the weight over
 * `ranks` ranks and the peers compute behind it: bounds[0] = 0 <
 * bounds[1] < ... < bounds[*pieces] = k.  `bounds` holds
 * HEXIR_SHARD_MAX_WEIGHT_PIECES + 1 entries.  One piece for one rank or
 * k < 2048; else [0, 512) and [512, k). */
hexir_status_t hexir_shard_weight_pieces(uint32_t k, uint32_t ranks,
                                         uint32_t *bounds, uint32_t *pieces);

typedef struct hexir_comm_t hexir_comm_t;

#define HEXIR_COMM_ID_BYTES 128

/* A fresh NCCL unique id (HEXIR_COMM_ID_BYTES bytes) for rank 0 to share. */
hexir_status_t hexir_comm_unique_id(void *id, size_t size);

/* Join a communicator of `nranks` processes as `rank`, driving GPU
 * `ordinal`.  Collective; also checks once whether the peers can map rank
 * 0's memory for direct row stores. */
hexir_status_t hexir_comm_init_rank(const void *id, size_t size, int nranks,
                                    int rank, int ordinal, hexir_comm_t **out);
void hexir_comm_release(hexir_comm_t *comm);
int hexir_comm_rank(const hexir_comm_t *comm);
int hexir_comm_size(const hexir_comm_t *comm);
/* 1 when the set-up check found that every peer can map rank 0's memory, so
 * hexir_sharded_linear_f64 can store rows into the root's c directly. */
int hexir_comm_direct_stores(const hexir_comm_t *comm);

/* Rank 0's flag: gather the rows with NCCL send/receive even where they
 * could be stored into its c directly. */
#define HEXIR_SHARD_GATHER_NCCL 0x1000u

/* Collective over all ranks of `comm` (rank 0 is the root):
 *   w      [k x n] on every rank; the root's contents are broadcast into the
 *          others' buffers.
 *   a_rows this rank's rows of a, rows hexir_shard_rows(m, size, rank).
 *   c      root: the whole [m x n] output; other ranks: [rows x n] staging
 *          for their own rows (partial sums, or rows that travel by NCCL;
 *          its contents are unspecified afterwards).
 * flags: HEXIR_MATMUL_RELU as for hexir_cuda_matmul_f64, HEXIR_SHARD_GATHER_NCCL.
 *
 * Rows go to the root's c directly when hexir_comm_init_rank found that
 * every peer can map rank 0's memory (same host, CUDA IPC) and the root's c
 * is exportable (a cuMemAlloc / cudaMalloc allocation); the root's stream
 * continues after every peer's kernel has finished storing.  Then, for
 * k >= 2048, w is broadcast in two k pieces (512, rest) and a peer computes
 * each piece as it lands, continuing its sums in its staging c, so only the
 * first piece's transfer is exposed; the result has the bits of one launch
 * over the rank's rows.  Otherwise rows are gathered with NCCL on a side
 * stream, piece by piece behind the GEMM.
 * Asynchronous on `stream`, except that with direct stores a peer's call
 * returns only once the root's stream has reached the same call (the root
 * sends the location of c every call).  Peers write the root's c only after
 * the root's `stream` reaches the call, so the root orders its own use of c
 * on that stream.
 *
 * Errors.  The return value reports this rank's own failures (a launch, a
 * driver or NCCL call).  A rank that fails still takes every collective step
 * of the call, so its peers never wait for ever, and marks a failure word
 * that every call max-reduces over all ranks on `stream`.  So the root's call
 * can return HEXIR_OK while a peer's rows were never written: before using
 * c, call hexir_comm_synchronize, which reports a failure on any rank. */
hexir_status_t hexir_sharded_linear_f64(hexir_comm_t *comm, const double *a_rows,
                                        double *w, double *c, uint32_t m,
                                        uint32_t n, uint32_t k, uint32_t flags,
                                        void *stream);

/* hexir_sharded_linear_host_f64 flag: every rank passes the whole weight
 * (the same values) and uploads only its share of its rows. */
#define HEXIR_SHARD_W_ON_ALL 0x4000u

/* The row-sharded linear with HOST buffers, for one process per GPU: the
 * call a program makes when its operands and result live in host memory.
 * Collective over all ranks of `comm`:
 *   a_rows  this rank's rows of a [rows x k], rows = hexir_shard_rows(m,
 *           size, rank);
 *   w       [k x n] on the root; with HEXIR_SHARD_W_ON_ALL on every rank
 *           (NULL elsewhere is allowed);
 *   c_rows  where this rank's rows of c [rows x n] go.
 * flags: HEXIR_MATMUL_RELU, HEXIR_SHARD_W_ON_ALL.
 *
 * Each rank moves its own rows over its own host link, so the copies of
 * all ranks run side by side, and the weight crosses a host link once: the
 * root uploads it and broadcasts it over NVLink, or, with
 * HEXIR_SHARD_W_ON_ALL, every rank uploads its share of it
 * (hexir_shard_rows over each piece's rows) and the shares meet over
 * NVLink.  For k >= 2048 the first half of k goes in growing pieces, and a
 * rank whose plan does not split k computes each piece over all its rows
 * as it lands (the rows' columns of that piece uploading beside it),
 * continuing its sums; the rest of k then runs per row chunk, and each
 * chunk downloads into c_rows while the next computes.  To hold the whole result in
 * one process, pass each rank a pointer into one shared mapping (rank r at
 * row hexir_shard_rows(m, size, r)).  Host memory that is page-locked
 * (hexir_host_register, or cuMemHostAlloc) moves at copy-engine speed;
 * pageable memory works, slower.  Each chunk runs the k split of one launch
 * over the rank's rows, so c_rows holds that launch's bits.  Device
 * workspace is kept in `comm` between calls.
 *
 * Synchronous: returns once this rank's rows are in c_rows, with
 * HEXIR_ERROR_DEVICE on every rank if any rank's part failed (as
 * hexir_comm_synchronize reports), HEXIR_ERROR_OUT_OF_MEMORY on every rank
 * if any rank could not get its workspace.  `stream` orders the call after
 * the caller's work on it. */
hexir_status_t hexir_sharded_linear_host_f64(hexir_comm_t *comm,
                                             const double *a_rows,
                                             const double *w, double *c_rows,
                                             uint32_t m, uint32_t n, uint32_t k,
                                             uint32_t flags, void *stream);

/* Page-lock (and unlock) an existing host range for fast copies to and from
 * every GPU of the process (cuMemHostRegister, portable), in the calling
 * thread's current CUDA context, or GPU 0's where none is current. */
hexir_status_t hexir_host_register(void *ptr, size_t bytes);
hexir_status_t hexir_host_unregister(void *ptr);

/* Waits for `stream` and returns HEXIR_ERROR_DEVICE on every rank if any
 * rank's part of any hexir_sharded_linear_f64 call on `comm` failed since
 * the last hexir_comm_synchronize (or a kernel on this GPU reported a device
 * error); HEXIR_OK otherwise.  Clears the failure.  Call it on every rank at
 * the same point of the call sequence, on the stream the calls used. */
hexir_status_t hexir_comm_synchronize(hexir_comm_t *comm, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_B200_COMM_H */
