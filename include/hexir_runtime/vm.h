/*
 * vm.h -- execute an entry point of a loaded module.
 *
 * hexir_execute and hexir_execute_capture keep the reference signatures and
 * meaning (runtime/include/hexir_runtime/vm.h:13-24): replay the entry's
 * command list; the capture variant copies the destination of the last
 * DISPATCH into `out_result`.
 *
 * Differences from the reference interpreter (runtime/src/vm/interpreter.c),
 * all of them additive:
 *   - a program may mix cpu- and cuda-placed kernels.  With a CUDA device the
 *     cpu-placed kernels run on the host and values move between host and GPU
 *     where the placement changes.  With a CPU device, cuda-placed kernels are
 *     refused exactly as before ("placed on cuda but the active device is
 *     cpu"): there is no host fallback for a cuda-placed kernel.
 *   - hexir_execute_devices runs a program whose kernels are placed on
 *     several GPUs ("cuda:N") or row-sharded over a range of them.
 */
#ifndef HEXIR_RUNTIME_VM_H
#define HEXIR_RUNTIME_VM_H

#include <stddef.h>

#include "hexir_runtime/hal.h"
#include "hexir_runtime/module.h"

#ifdef __cplusplus
extern "C" {
#endif

hexir_status_t hexir_execute(const hexir_module_t *module,
                             hexir_device_t *device, const char *entry);

hexir_status_t hexir_execute_capture(const hexir_module_t *module,
                                     hexir_device_t *device, const char *entry,
                                     void *out_result, size_t out_size);

/* extension: run with a set of CUDA devices; devices[i] serves "cuda:i".
 * A kernel placed on cuda:N needs N < device_count; a row-sharded kernel
 * needs its whole ordinal range.  cpu-placed kernels run on the host.  Row
 * sharding uses NCCL (libnccl.so.2, loaded on first use) to broadcast the
 * weight from the first device of the range and to gather the output rows
 * back to it. */
hexir_status_t hexir_execute_devices(const hexir_module_t *module,
                                     hexir_device_t *const *devices,
                                     unsigned device_count, const char *entry,
                                     void *out_result, size_t out_size);

/* extension: device time of the kernels of the last execute on this thread,
 * in milliseconds, summed over dispatches (CUDA events around each DISPATCH
 * on the launching stream).  0 when nothing ran on a GPU. */
double hexir_last_execute_kernel_ms(void);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_RUNTIME_VM_H */
