/*
 * hexir_b200/fault.h -- host-side fault injection, for tests of the error
 * paths.  No counterpart in the reference runtime, which reports failures
 * but offers no way to cause them (runtime/src/hal/cuda/cuda_device.c:62-68).
 *
 * A rule names a site and the calls at it that fail:
 *
 *   alloc:N     the N-th allocation fails with HEXIR_ERROR_OUT_OF_MEMORY
 *               (host slot storage of the VM, HAL buffers on either device,
 *               a kept constant -- which then falls back to a per-execute
 *               upload -- and the split-K workspace)
 *   launch:N    the N-th kernel launch fails with HEXIR_ERROR_DEVICE before
 *               reaching the driver
 *   nccl:N      the N-th grouped NCCL step of a row-sharded dispatch in one
 *               process (weight broadcast, row gather) fails with
 *               HEXIR_ERROR_DEVICE before any rank enqueues it
 *
 * "site:N+" fails the N-th call and every later one.  Rules are separated by
 * commas: "alloc:3,launch:1+".  Counting starts when the rules are set.  The
 * multi-process entry points (comm.h) take no injected NCCL faults: a rank
 * failing alone would leave its peers' collectives waiting on the GPU.
 *
 * The environment variable HEXIR_FAULT holds rules read at the first check in
 * the process; hexir_fault_configure replaces them.
 */
#ifndef HEXIR_B200_FAULT_H
#define HEXIR_B200_FAULT_H

#include <stdint.h>

#include "hexir_runtime/status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Replace the rules (NULL or "" turns injection off) and restart the call
 * counts.  A malformed spec returns HEXIR_ERROR_INVALID_ARGUMENT and leaves
 * the previous rules in force. */
hexir_status_t hexir_fault_configure(const char *spec);

/* Calls counted at `site` ("alloc", "launch", "nccl") since the rules were
 * set; 0 while injection is off or for an unknown site. */
uint64_t hexir_fault_calls(const char *site);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_B200_FAULT_H */
