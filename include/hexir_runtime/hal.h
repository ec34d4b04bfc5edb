/*
 * hal.h -- the device boundary of the hexir runtime.
 *
 * Every function the reference declares in runtime/include/hexir_runtime/hal.h
 * (lines 22-83) is declared here with the same name, signature and meaning, so
 * a program written against the reference HAL links against this library
 * unchanged.  The CUDA backend behind it is new: primary context per GPU, one
 * stream per device, asynchronous launches, a cached kernel module per device,
 * and the sm_100a kernels of this project.
 *
 * Additions (marked "extension") give a program more than GPU 0:
 * hexir_device_create_cuda(ordinal) opens a particular GPU, and
 * hexir_device_count reports how many there are.
 */
#ifndef HEXIR_RUNTIME_HAL_H
#define HEXIR_RUNTIME_HAL_H

#include <stddef.h>
#include <stdint.h>

#include "hexir_runtime/status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  HEXIR_DEVICE_CPU = 0,
  HEXIR_DEVICE_CUDA = 1,
} hexir_device_kind_t;

typedef struct hexir_device_t hexir_device_t;
typedef struct hexir_buffer_t hexir_buffer_t;

typedef enum {
  HEXIR_MEMORY_HOST_LOCAL = 0,   /* ordinary host RAM */
  HEXIR_MEMORY_DEVICE_LOCAL = 1, /* device RAM; reach it with write/read */
  HEXIR_MEMORY_HOST_VISIBLE = 2, /* addressable from the host directly */
} hexir_memory_kind_t;

/* Open a device.  HEXIR_DEVICE_CUDA opens GPU 0 (reference hal.h:39). */
hexir_status_t hexir_device_create(hexir_device_kind_t kind,
                                   hexir_device_t **out_device);
void hexir_device_release(hexir_device_t *device);
const char *hexir_device_name(const hexir_device_t *device);
hexir_device_kind_t hexir_device_kind(const hexir_device_t *device);

/* Wait until all work submitted to the device has finished.  Returns
 * HEXIR_ERROR_DEVICE if a kernel reported a failure (for example a pipeline
 * wait that ran out of its iteration budget). */
hexir_status_t hexir_device_wait(hexir_device_t *device);

hexir_status_t hexir_buffer_allocate(hexir_device_t *device, size_t size,
                                     hexir_memory_kind_t memory,
                                     hexir_buffer_t **out_buffer);
void hexir_buffer_release(hexir_buffer_t *buffer);
size_t hexir_buffer_size(const hexir_buffer_t *buffer);
hexir_memory_kind_t hexir_buffer_memory_kind(const hexir_buffer_t *buffer);

/* NULL for DEVICE_LOCAL buffers. */
void *hexir_buffer_host_pointer(hexir_buffer_t *buffer);

/* The backend's own address: a CUdeviceptr for CUDA, a host pointer for CPU. */
void *hexir_buffer_device_pointer(hexir_buffer_t *buffer);

/* Host to buffer copy of `size` bytes (size <= buffer size).  The source may
 * be reused as soon as the call returns. */
hexir_status_t hexir_buffer_write(hexir_buffer_t *dst, const void *src,
                                  size_t size);
/* Buffer to host copy; waits for the work that produces the buffer. */
hexir_status_t hexir_buffer_read(const hexir_buffer_t *src, void *dst,
                                 size_t size);

/* Launch kernel `entry` of a device image with one device pointer per buffer
 * (the reference's bare-pointer convention, hal.h:70-83).  UNIMPLEMENTED on
 * the CPU backend.  Modules produced for this library carry a LAUNCH section
 * and are launched by the VM through the kernel library instead
 * (hexir_b200/kernels.h); this entry point serves images that follow the
 * reference convention. */
hexir_status_t hexir_device_launch(hexir_device_t *device, const void *image,
                                   size_t image_size, const char *entry,
                                   unsigned grid_x, unsigned grid_y,
                                   unsigned block_x, unsigned block_y,
                                   hexir_buffer_t **args, unsigned arg_count);

/* extension: open CUDA device `ordinal` ("cuda:N").  Ordinal 0 is what
 * hexir_device_create(HEXIR_DEVICE_CUDA) opens. */
hexir_status_t hexir_device_create_cuda(int ordinal,
                                        hexir_device_t **out_device);

/* extension: CUDA ordinal of a device (-1 for the CPU device). */
int hexir_device_ordinal(const hexir_device_t *device);

/* extension: number of devices of `kind` (CPU: 1; CUDA: 0 if no driver). */
hexir_status_t hexir_device_count(hexir_device_kind_t kind, int *out_count);

/* extension: the CUstream the device submits work on (NULL for CPU). */
void *hexir_device_stream(hexir_device_t *device);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_RUNTIME_HAL_H */
