/*
 * hexir_b200/comm.h -- row sharding of a linear across GPUs.
 *
 * The reference has no multi-GPU path; its placement is per op and per
 * process (compiler/Target/TargetInfo.cpp:20-45, runtime/src/vm/
 * interpreter.c:85-92).  This header adds the one strategy the hot path
 * needs: the rows of a[m x k] (and so of c[m x n]) are split over GPUs, the
 * weight b[k x n] is broadcast from the first GPU over NVLink with NCCL, every
 * GPU computes its rows with no collective, and the output rows are gathered
 * back to the first GPU.
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

typedef struct hexir_comm_t hexir_comm_t;

#define HEXIR_COMM_ID_BYTES 128

/* A fresh NCCL unique id (HEXIR_COMM_ID_BYTES bytes) for rank 0 to share. */
hexir_status_t hexir_comm_unique_id(void *id, size_t size);

/* Join a communicator of `nranks` processes as `rank`, driving GPU
 * `ordinal`. */
hexir_status_t hexir_comm_init_rank(const void *id, size_t size, int nranks,
                                    int rank, int ordinal, hexir_comm_t **out);
void hexir_comm_release(hexir_comm_t *comm);
int hexir_comm_rank(const hexir_comm_t *comm);
int hexir_comm_size(const hexir_comm_t *comm);

/* Collective over all ranks of `comm` (rank 0 is the root):
 *   w      [k x n] on every rank; the root's contents are broadcast into the
 *          others' buffers.
 *   a_rows this rank's rows of a, rows hexir_shard_rows(m, size, rank).
 *   c      root: the whole [m x n] output; other ranks: [rows x n] for their
 *          own rows, which are then sent to the root.
 * flags: HEXIR_MATMUL_RELU as for hexir_cuda_matmul_f64.  Asynchronous on
 * `stream`. */
hexir_status_t hexir_sharded_linear_f64(hexir_comm_t *comm, const double *a_rows,
                                        double *w, double *c, uint32_t m,
                                        uint32_t n, uint32_t k, uint32_t flags,
                                        void *stream);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_B200_COMM_H */
