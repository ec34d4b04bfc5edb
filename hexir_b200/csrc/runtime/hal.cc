// hal.cc -- public HAL entry points (include/hexir_runtime/hal.h) and the CPU
// and CUDA backends.
//
// Entry-point semantics follow the reference runtime/src/hal/hal.c:7-103
// (argument checks, size checks on write/read, UNIMPLEMENTED launch on CPU).
// The CUDA backend differs from runtime/src/hal/cuda/cuda_device.c by design:
// primary context per ordinal instead of a fresh context on device 0, one
// non-blocking stream per device object, launches that do not synchronise,
// and cached modules for images launched by name.

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include "cuda_driver.h"
#include "fault.h"
#include "hal_internal.h"
#include "kernel_lib.h"

namespace hexir {

void report(const std::string &message) {
  std::fprintf(stderr, "hexir: %s\n", message.c_str());
}

namespace {

// ---- CPU backend: host memory, synchronous by construction ---------------

struct CpuDevice : hexir_device_t {
  CpuDevice() {
    kind = HEXIR_DEVICE_CPU;
    name = "cpu";
  }
  hexir_status_t buffer_allocate(size_t size, hexir_memory_kind_t,
                                 hexir_buffer_t **out) override {
    if (fault_hit(FaultSite::Alloc))
      return HEXIR_ERROR_OUT_OF_MEMORY;
    auto *buffer = new (std::nothrow) hexir_buffer_t;
    if (!buffer)
      return HEXIR_ERROR_OUT_OF_MEMORY;
    void *data = size ? std::calloc(1, size) : nullptr;
    if (size && !data) {
      delete buffer;
      return HEXIR_ERROR_OUT_OF_MEMORY;
    }
    buffer->device = this;
    buffer->size = size;
    buffer->memory = HEXIR_MEMORY_HOST_VISIBLE;
    buffer->impl = data;
    *out = buffer;
    return HEXIR_OK;
  }
  void buffer_release(hexir_buffer_t *buffer) override {
    std::free(buffer->impl);
    delete buffer;
  }
  hexir_status_t buffer_write(hexir_buffer_t *dst, const void *src,
                              size_t size) override {
    if (size)
      std::memcpy(dst->impl, src, size);
    return HEXIR_OK;
  }
  hexir_status_t buffer_read(const hexir_buffer_t *src, void *dst,
                             size_t size) override {
    if (size)
      std::memcpy(dst, src->impl, size);
    return HEXIR_OK;
  }
  void *buffer_host_pointer(hexir_buffer_t *buffer) override {
    return buffer->impl;
  }
  hexir_status_t wait() override { return HEXIR_OK; }
};

// Modules of images launched by entry name (the reference's bare-pointer
// convention), cached per (context, image content).
std::mutex g_named_mu;
std::map<std::pair<CUcontext, uint64_t>, CUmodule> g_named_modules;

}  // namespace

namespace {
std::mutex g_pinned_mu;
std::multimap<size_t, void *> g_pinned;  // free blocks by size
size_t g_pinned_bytes = 0;
constexpr size_t kPinnedCapBytes = 8ull << 30;
}  // namespace

void *pinned_take(size_t bytes, CUcontext context) {
  if (!bytes)
    return nullptr;
  {
    std::lock_guard<std::mutex> lock(g_pinned_mu);
    auto it = g_pinned.find(bytes);
    if (it != g_pinned.end()) {
      void *p = it->second;
      g_pinned.erase(it);
      g_pinned_bytes -= bytes;
      return p;
    }
  }
  const Driver &d = driver();
  if (!d.ok)
    return nullptr;
  ContextGuard guard(context);
  void *p = nullptr;
  if (d.MemHostAlloc(&p, bytes, CU_MEMHOSTALLOC_PORTABLE) != CUDA_SUCCESS)
    return nullptr;
  return p;
}

void pinned_give(void *block, size_t bytes) {
  if (!block)
    return;
  {
    std::lock_guard<std::mutex> lock(g_pinned_mu);
    if (g_pinned_bytes + bytes <= kPinnedCapBytes) {
      g_pinned.emplace(bytes, block);
      g_pinned_bytes += bytes;
      return;
    }
  }
  driver().MemFreeHost(block);
}

CudaDevice *as_cuda(hexir_device_t *device) {
  return device && device->kind == HEXIR_DEVICE_CUDA
             ? static_cast<CudaDevice *>(device)
             : nullptr;
}

CUstream CudaDevice::copy_stream() {
  if (!copies) {
    ContextGuard guard(state->context);
    if (driver().StreamCreate(&copies, CU_STREAM_NON_BLOCKING) != CUDA_SUCCESS)
      copies = nullptr;
  }
  return copies;
}

CUstream CudaDevice::side_stream() {
  if (!side) {
    ContextGuard guard(state->context);
    if (driver().StreamCreate(&side, CU_STREAM_NON_BLOCKING) != CUDA_SUCCESS)
      side = nullptr;
  }
  return side;
}

CudaDevice::~CudaDevice() {
  if (side) {
    ContextGuard guard(state->context);
    driver().StreamSynchronize(side);
    driver().StreamDestroy(side);
  }
  if (copies) {
    ContextGuard guard(state->context);
    driver().StreamSynchronize(copies);
    driver().StreamDestroy(copies);
  }
  if (stream) {
    ContextGuard guard(state->context);
    driver().StreamSynchronize(stream);
    std::lock_guard<std::mutex> lock(pool_mu);
    for (auto &kv : pool)
      driver().MemFree(kv.second);
    pool.clear();
    driver().StreamDestroy(stream);
  }
}

hexir_status_t CudaDevice::allocate_pooled(size_t size, hexir_buffer_t **out) {
  std::lock_guard<std::mutex> lock(pool_mu);
  auto it = pool.find(size);
  if (it == pool.end()) {
    hexir_status_t st = allocate_raw(size, out);
    if (st == HEXIR_ERROR_OUT_OF_MEMORY && !pool.empty()) {
      // Give the pool back and try once more.
      ContextGuard guard(state->context);
      driver().StreamSynchronize(stream);
      for (auto &kv : pool)
        driver().MemFree(kv.second);
      pool.clear();
      pool_bytes = 0;
      st = allocate_raw(size, out);
    }
    if (st == HEXIR_OK)
      (*out)->pooled = true;
    return st;
  }
  auto *buffer = new (std::nothrow) hexir_buffer_t;
  if (!buffer)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  buffer->device = this;
  buffer->size = size;
  buffer->memory = HEXIR_MEMORY_DEVICE_LOCAL;
  buffer->impl = reinterpret_cast<void *>(static_cast<uintptr_t>(it->second));
  buffer->pooled = true;
  pool_bytes -= size;
  pool.erase(it);
  *out = buffer;
  return HEXIR_OK;
}

hexir_status_t CudaDevice::allocate_raw(size_t size, hexir_buffer_t **out) {
  const Driver &d = driver();
  if (fault_hit(FaultSite::Alloc)) {
    report("cuMemAlloc(" + std::to_string(size) + "): injected fault (HEXIR_FAULT)");
    return HEXIR_ERROR_OUT_OF_MEMORY;
  }
  auto *buffer = new (std::nothrow) hexir_buffer_t;
  if (!buffer)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  CUdeviceptr ptr = 0;
  if (size) {
    ContextGuard guard(state->context);
    CUresult r = d.MemAlloc(&ptr, size);
    if (r != CUDA_SUCCESS) {
      report("cuMemAlloc(" + std::to_string(size) + ") failed: " +
             cuda_message("cuMemAlloc", r));
      delete buffer;
      return HEXIR_ERROR_OUT_OF_MEMORY;
    }
  }
  buffer->device = this;
  buffer->size = size;
  buffer->memory = HEXIR_MEMORY_DEVICE_LOCAL;
  buffer->impl = reinterpret_cast<void *>(static_cast<uintptr_t>(ptr));
  *out = buffer;
  return HEXIR_OK;
}

hexir_status_t CudaDevice::buffer_allocate(size_t size, hexir_memory_kind_t,
                                           hexir_buffer_t **out) {
  hexir_status_t s = allocate_raw(size, out);
  if (s != HEXIR_OK || size == 0)
    return s;
  // The program format promises zeroed ALLOC buffers (program.h).
  ContextGuard guard(state->context);
  CUresult r = driver().MemsetD8Async(
      reinterpret_cast<CUdeviceptr>((*out)->impl), 0, size, stream);
  if (r != CUDA_SUCCESS) {
    report(cuda_message("cuMemsetD8Async", r));
    buffer_release(*out);
    *out = nullptr;
    return HEXIR_ERROR_DEVICE;
  }
  return HEXIR_OK;
}

void CudaDevice::buffer_release(hexir_buffer_t *buffer) {
  if (buffer->borrowed) {
    delete buffer;
    return;
  }
  // The pool keeps at most kPoolCapBytes; beyond that blocks are freed.
  constexpr size_t kPoolCapBytes = 32ull << 30;
  if (buffer->pooled && buffer->impl) {
    std::lock_guard<std::mutex> lock(pool_mu);
    if (pool_bytes + buffer->size <= kPoolCapBytes) {
      pool.emplace(buffer->size, reinterpret_cast<CUdeviceptr>(buffer->impl));
      pool_bytes += buffer->size;
      delete buffer;
      return;
    }
  }
  if (buffer->impl) {
    ContextGuard guard(state->context);
    // Work queued on this stream may still use the buffer.
    driver().StreamSynchronize(stream);
    driver().MemFree(reinterpret_cast<CUdeviceptr>(buffer->impl));
  }
  delete buffer;
}

hexir_status_t CudaDevice::write_async(CUdeviceptr dst, const void *src,
                                       size_t size) {
  if (!size)
    return HEXIR_OK;
  ContextGuard guard(state->context);
  CUresult r = driver().MemcpyHtoDAsync(dst, src, size, stream);
  if (r != CUDA_SUCCESS) {
    report("host to device copy failed: " + cuda_message("cuMemcpyHtoDAsync", r));
    return HEXIR_ERROR_DEVICE;
  }
  return HEXIR_OK;
}

hexir_status_t CudaDevice::buffer_write(hexir_buffer_t *dst, const void *src,
                                        size_t size) {
  hexir_status_t s =
      write_async(reinterpret_cast<CUdeviceptr>(dst->impl), src, size);
  if (s != HEXIR_OK)
    return s;
  // Synchronous like the reference: the caller may then free `src` even if it
  // is pinned memory.
  ContextGuard guard(state->context);
  CUresult r = driver().StreamSynchronize(stream);
  if (r != CUDA_SUCCESS) {
    report("host to device copy failed: " + cuda_message("cuStreamSynchronize", r));
    return HEXIR_ERROR_DEVICE;
  }
  return HEXIR_OK;
}

hexir_status_t CudaDevice::buffer_read(const hexir_buffer_t *src, void *dst,
                                       size_t size) {
  if (!size)
    return HEXIR_OK;
  ContextGuard guard(state->context);
  CUresult r = driver().MemcpyDtoHAsync(
      dst, reinterpret_cast<CUdeviceptr>(src->impl), size, stream);
  if (r == CUDA_SUCCESS)
    r = driver().StreamSynchronize(stream);
  if (r != CUDA_SUCCESS) {
    report("device to host copy failed: " + cuda_message("cuMemcpyDtoHAsync", r));
    return HEXIR_ERROR_DEVICE;
  }
  std::string error;
  if (check_device(state, stream, &error) != HEXIR_OK) {
    report(error);
    return HEXIR_ERROR_DEVICE;
  }
  return HEXIR_OK;
}

hexir_status_t CudaDevice::launch(const void *image, size_t image_size,
                                  const char *entry, unsigned grid_x,
                                  unsigned grid_y, unsigned block_x,
                                  unsigned block_y, hexir_buffer_t **args,
                                  unsigned arg_count) {
  const Driver &d = driver();
  enum { kMaxArgs = 8 };
  if (arg_count > kMaxArgs)
    return HEXIR_ERROR_INVALID_MODULE;
  ContextGuard guard(state->context);
  CUmodule module = nullptr;
  {
    const auto key = std::make_pair(state->context, hash_bytes(image, image_size));
    std::lock_guard<std::mutex> lock(g_named_mu);
    auto it = g_named_modules.find(key);
    if (it != g_named_modules.end()) {
      module = it->second;
    } else {
      CUresult r = d.ModuleLoadData(&module, image);
      if (r != CUDA_SUCCESS) {
        report("cannot load device image: " + cuda_message("cuModuleLoadData", r));
        return HEXIR_ERROR_DEVICE;
      }
      g_named_modules[key] = module;
    }
  }
  CUfunction function = nullptr;
  CUresult r = d.ModuleGetFunction(&function, module, entry);
  if (r != CUDA_SUCCESS) {
    report(std::string("no kernel '") + entry + "' in the device image: " +
           cuda_message("cuModuleGetFunction", r));
    return HEXIR_ERROR_NOT_FOUND;
  }
  CUdeviceptr addresses[kMaxArgs];
  void *params[kMaxArgs];
  for (unsigned i = 0; i < arg_count; ++i) {
    addresses[i] = reinterpret_cast<CUdeviceptr>(args[i]->impl);
    params[i] = &addresses[i];
  }
  if (fault_hit(FaultSite::Launch)) {
    report(std::string("launch of '") + entry + "': injected fault (HEXIR_FAULT)");
    return HEXIR_ERROR_DEVICE;
  }
  r = d.LaunchKernel(function, grid_x, grid_y, 1, block_x, block_y, 1, 0, stream,
                     params, nullptr);
  if (r != CUDA_SUCCESS) {
    report(std::string("launch of '") + entry + "' failed: " +
           cuda_message("cuLaunchKernel", r));
    return HEXIR_ERROR_DEVICE;
  }
  count_launch();
  return HEXIR_OK;
}

hexir_status_t CudaDevice::wait() {
  std::string error;
  if (check_device(state, stream, &error) != HEXIR_OK) {
    report("device synchronize failed: " + error);
    return HEXIR_ERROR_DEVICE;
  }
  return HEXIR_OK;
}

static hexir_status_t create_cuda(int ordinal, hexir_device_t **out) {
  std::string error;
  DeviceState *state = device_state(ordinal, &error);
  if (!state) {
    report(error);
    return HEXIR_ERROR_DEVICE;
  }
  auto *device = new (std::nothrow) CudaDevice;
  if (!device)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  device->kind = HEXIR_DEVICE_CUDA;
  device->ordinal = ordinal;
  device->state = state;
  device->name = "cuda";
  if (ordinal != 0)
    device->name += ":" + std::to_string(ordinal);
  if (!state->name.empty())
    device->name += " (" + state->name + ")";
  ContextGuard guard(state->context);
  CUresult r = driver().StreamCreate(&device->stream, CU_STREAM_NON_BLOCKING);
  if (r != CUDA_SUCCESS) {
    report(cuda_message("cuStreamCreate", r));
    delete device;
    return HEXIR_ERROR_DEVICE;
  }
  *out = device;
  return HEXIR_OK;
}

}  // namespace hexir

using namespace hexir;

extern "C" {

hexir_status_t hexir_device_create(hexir_device_kind_t kind,
                                   hexir_device_t **out_device) {
  if (!out_device)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out_device = nullptr;
  switch (kind) {
  case HEXIR_DEVICE_CPU: {
    auto *device = new (std::nothrow) CpuDevice;
    if (!device)
      return HEXIR_ERROR_OUT_OF_MEMORY;
    *out_device = device;
    return HEXIR_OK;
  }
  case HEXIR_DEVICE_CUDA:
    return create_cuda(0, out_device);
  }
  return HEXIR_ERROR_INVALID_ARGUMENT;
}

hexir_status_t hexir_device_create_cuda(int ordinal,
                                        hexir_device_t **out_device) {
  if (!out_device || ordinal < 0)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out_device = nullptr;
  return create_cuda(ordinal, out_device);
}

void hexir_device_release(hexir_device_t *device) { delete device; }

const char *hexir_device_name(const hexir_device_t *device) {
  return device ? device->name.c_str() : "(null)";
}

hexir_device_kind_t hexir_device_kind(const hexir_device_t *device) {
  return device ? device->kind : HEXIR_DEVICE_CPU;
}

int hexir_device_ordinal(const hexir_device_t *device) {
  return device ? device->ordinal : -1;
}

hexir_status_t hexir_device_count(hexir_device_kind_t kind, int *out_count) {
  if (!out_count)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out_count = 0;
  if (kind == HEXIR_DEVICE_CPU) {
    *out_count = 1;
    return HEXIR_OK;
  }
  const Driver &d = driver();
  if (!d.ok)
    return HEXIR_OK;
  int count = 0;
  if (d.DeviceGetCount(&count) == CUDA_SUCCESS)
    *out_count = count;
  return HEXIR_OK;
}

void *hexir_device_stream(hexir_device_t *device) {
  CudaDevice *cuda = as_cuda(device);
  return cuda ? static_cast<void *>(cuda->stream) : nullptr;
}

hexir_status_t hexir_device_wait(hexir_device_t *device) {
  if (!device)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  return device->wait();
}

hexir_status_t hexir_buffer_allocate(hexir_device_t *device, size_t size,
                                     hexir_memory_kind_t memory,
                                     hexir_buffer_t **out_buffer) {
  if (!device || !out_buffer)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out_buffer = nullptr;
  return device->buffer_allocate(size, memory, out_buffer);
}

void hexir_buffer_release(hexir_buffer_t *buffer) {
  if (buffer && buffer->device)
    buffer->device->buffer_release(buffer);
}

size_t hexir_buffer_size(const hexir_buffer_t *buffer) {
  return buffer ? buffer->size : 0u;
}

hexir_memory_kind_t hexir_buffer_memory_kind(const hexir_buffer_t *buffer) {
  return buffer ? buffer->memory : HEXIR_MEMORY_HOST_LOCAL;
}

void *hexir_buffer_host_pointer(hexir_buffer_t *buffer) {
  return buffer ? buffer->device->buffer_host_pointer(buffer) : nullptr;
}

void *hexir_buffer_device_pointer(hexir_buffer_t *buffer) {
  return buffer ? buffer->impl : nullptr;
}

hexir_status_t hexir_buffer_write(hexir_buffer_t *dst, const void *src,
                                  size_t size) {
  if (!dst || !src)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  if (size > dst->size)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  return dst->device->buffer_write(dst, src, size);
}

hexir_status_t hexir_buffer_read(const hexir_buffer_t *src, void *dst,
                                 size_t size) {
  if (!src || !dst)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  if (size > src->size)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  return src->device->buffer_read(src, dst, size);
}

hexir_status_t hexir_device_launch(hexir_device_t *device, const void *image,
                                   size_t image_size, const char *entry,
                                   unsigned grid_x, unsigned grid_y,
                                   unsigned block_x, unsigned block_y,
                                   hexir_buffer_t **args, unsigned arg_count) {
  if (!device || !image || !entry)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  return device->launch(image, image_size, entry, grid_x, grid_y, block_x,
                        block_y, args, arg_count);
}

const char *hexir_status_string(hexir_status_t status) {
  switch (status) {
  case HEXIR_OK: return "ok";
  case HEXIR_ERROR_INVALID_ARGUMENT: return "invalid argument";
  case HEXIR_ERROR_NOT_FOUND: return "not found";
  case HEXIR_ERROR_OUT_OF_MEMORY: return "out of memory";
  case HEXIR_ERROR_UNIMPLEMENTED: return "unimplemented";
  case HEXIR_ERROR_INVALID_MODULE: return "invalid module";
  case HEXIR_ERROR_IO: return "io error";
  case HEXIR_ERROR_DEVICE: return "device error";
  }
  return "unknown";
}

}  // extern "C"
