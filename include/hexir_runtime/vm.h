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
 * weight from the first device of the range; the output rows land on that
 * device through peer stores from each GPU's kernel (NCCL send/receive where
 * peer access is unavailable). */
hexir_status_t hexir_execute_devices(const hexir_module_t *module,
                                     hexir_device_t *const *devices,
                                     unsigned device_count, const char *entry,
                                     void *out_result, size_t out_size);

/* extension: device time of the dispatches of the last execute on this
 * thread, in milliseconds, summed (CUDA events around each DISPATCH on the
 * launching stream).  A pipelined dispatch's span includes its waits on the
 * uploads it overlaps; with the constants kept on the GPU
 * (hexir_module_keep_constants) the spans are the kernels alone.  0 when
 * nothing ran on a GPU. */
double hexir_last_execute_kernel_ms(void);

/* extension: keep the module's constants on the device between executes.
 * With `enable` set, the first execute that needs a CONST on a GPU uploads it
 * into memory that stays with the module, and later executes of the module
 * on that GPU (through any device object, from any thread) read it there
 * instead of copying RODATA again; the reference re-uploads every constant
 * on every execute (runtime/src/vm/interpreter.c:300-315).  A dispatch
 * whose destination is a CONST slot writes a private buffer, never the kept
 * copy.  `enable` = 0 frees the kept copies (after the GPUs finish with
 * them), as does hexir_module_release; neither may overlap an execute of the
 * module on another thread.  Off by default. */
hexir_status_t hexir_module_keep_constants(hexir_module_t *module, int enable);

/* extension: bytes of constants currently kept on GPUs for `module`. */
size_t hexir_module_kept_bytes(const hexir_module_t *module);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_RUNTIME_VM_H */
