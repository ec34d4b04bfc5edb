// hal_internal.h -- backend interface behind include/hexir_runtime/hal.h.
//
// The reference keeps a C vtable per backend (runtime/src/hal/hal_internal.h);
// here each backend is a C++ class deriving from hexir_device_t.  The public
// structs stay opaque to C callers.
#pragma once

#include <cuda.h>

#include <cstddef>
#include <map>
#include <mutex>
#include <string>

#include "hexir_runtime/hal.h"

namespace hexir {
struct DeviceState;
}

struct hexir_device_t {
  hexir_device_kind_t kind = HEXIR_DEVICE_CPU;
  int ordinal = -1;
  std::string name;

  virtual ~hexir_device_t() = default;
  virtual hexir_status_t buffer_allocate(size_t size, hexir_memory_kind_t memory,
                                         hexir_buffer_t **out) = 0;
  virtual void buffer_release(hexir_buffer_t *buffer) = 0;
  virtual hexir_status_t buffer_write(hexir_buffer_t *dst, const void *src,
                                      size_t size) = 0;
  virtual hexir_status_t buffer_read(const hexir_buffer_t *src, void *dst,
                                     size_t size) = 0;
  virtual void *buffer_host_pointer(hexir_buffer_t *buffer) = 0;
  virtual hexir_status_t launch(const void *image, size_t image_size,
                                const char *entry, unsigned grid_x,
                                unsigned grid_y, unsigned block_x,
                                unsigned block_y, hexir_buffer_t **args,
                                unsigned arg_count) {
    (void)image; (void)image_size; (void)entry; (void)grid_x; (void)grid_y;
    (void)block_x; (void)block_y; (void)args; (void)arg_count;
    return HEXIR_ERROR_UNIMPLEMENTED;
  }
  virtual hexir_status_t wait() = 0;
};

struct hexir_buffer_t {
  hexir_device_t *device = nullptr;
  size_t size = 0;
  hexir_memory_kind_t memory = HEXIR_MEMORY_HOST_LOCAL;
  void *impl = nullptr;  // host pointer (CPU) or CUdeviceptr (CUDA)
  bool pooled = false;   // VM buffer: returns to the device's pool on release
  bool borrowed = false; // VM view of memory it does not own (a constant the
                         // module keeps on the device): release frees no memory
};

namespace hexir {

// The CUDA backend, visible to the VM for asynchronous copies and launches.
struct CudaDevice : hexir_device_t {
  DeviceState *state = nullptr;
  CUstream stream = nullptr;

  ~CudaDevice() override;
  hexir_status_t buffer_allocate(size_t size, hexir_memory_kind_t memory,
                                 hexir_buffer_t **out) override;
  void buffer_release(hexir_buffer_t *buffer) override;
  hexir_status_t buffer_write(hexir_buffer_t *dst, const void *src,
                              size_t size) override;
  hexir_status_t buffer_read(const hexir_buffer_t *src, void *dst,
                             size_t size) override;
  void *buffer_host_pointer(hexir_buffer_t *) override { return nullptr; }
  hexir_status_t launch(const void *image, size_t image_size, const char *entry,
                        unsigned grid_x, unsigned grid_y, unsigned block_x,
                        unsigned block_y, hexir_buffer_t **args,
                        unsigned arg_count) override;
  hexir_status_t wait() override;

  // Host to device copy on this device's stream; returns before the copy
  // completes (pageable sources are staged by the driver first).
  hexir_status_t write_async(CUdeviceptr dst, const void *src, size_t size);
  // Allocate without zeroing (the VM zeroes lazily where it must).
  hexir_status_t allocate_raw(size_t size, hexir_buffer_t **out);
  // Same, from the device's pool of released VM buffers when one of exactly
  // this size is free.  Pooled blocks are reused in stream order (every VM
  // use is on this device's stream), capped at 32 GiB per device, and freed
  // with the device.  `pool_mu` guards the pool itself; the VM still runs
  // one execute per device object at a time (its streams are the object's).
  hexir_status_t allocate_pooled(size_t size, hexir_buffer_t **out);

  std::mutex pool_mu;
  std::multimap<size_t, CUdeviceptr> pool;
  size_t pool_bytes = 0;

  // Second stream for copies that overlap the kernels on `stream` (the VM's
  // pipelined upload / download of a large dispatch); created on first use.
  CUstream copy_stream();
  CUstream copies = nullptr;

  // Second compute stream: independent row chunks of one dispatch alternate
  // between `stream` and this one, so one chunk's last wave of tiles
  // overlaps the next chunk's first; created on first use.
  CUstream side_stream();
  CUstream side = nullptr;
};

CudaDevice *as_cuda(hexir_device_t *device);

// Page-locked host blocks, kept across executes and shared by every device
// of the process: a module whose ops alternate between host and GPU copies
// whole tensors both ways every execute, and page-locked memory moves them
// at copy-engine speed without the driver's pageable staging.  take returns
// a block of exactly `bytes` (from the pool, else newly page-locked with
// `context` current; portable to every context), or nullptr when none can
// be had; give returns it once no copy can still use it.  At most 8 GiB
// stay pooled.
void *pinned_take(size_t bytes, CUcontext context);
void pinned_give(void *block, size_t bytes);

// Reports a backend failure the way the reference does: "hexir: <message>"
// on stderr.
void report(const std::string &message);

}  // namespace hexir

// CPU reference kernels used for cpu-placed dispatches (cpu_kernels.cc).
namespace hexir {
void cpu_matmul_f64(const double *a, const double *b, double *c, uint32_t m,
                    uint32_t n, uint32_t k);
void cpu_add_f64(const double *a, const double *b, double *c, size_t n);
void cpu_relu_f64(const double *x, double *y, size_t n);
// memcpy over the host threads (large copies between host buffers, e.g.
// out of page-locked staging into a caller's pageable memory).
void parallel_copy(void *dst, const void *src, size_t bytes);
// y = op(x) over a row-major [rows x cols] tensor for the activation kernel
// kinds 7-14 of program.h (softmax along each row).
void cpu_activation_f64(uint32_t kind, const double *x, double *y,
                        uint64_t rows, uint64_t cols);
}  // namespace hexir
