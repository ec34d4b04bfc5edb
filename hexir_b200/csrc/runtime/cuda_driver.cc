// cuda_driver.cc -- dlopen of libcuda and symbol binding (see cuda_driver.h).

#include "cuda_driver.h"

#include <dlfcn.h>

#include <mutex>

namespace hexir {

namespace {

Driver g_driver;
std::once_flag g_once;

template <typename Fn>
bool bind(void *lib, Fn &slot, const char *symbol, std::string &error) {
  void *p = dlsym(lib, symbol);
  if (!p) {
    error = std::string("libcuda is missing ") + symbol;
    return false;
  }
  slot = reinterpret_cast<Fn>(p);
  return true;
}

void load() {
  Driver &d = g_driver;
  // The driver's soname; the unversioned name is a toolkit symlink that a
  // machine with only the driver may not have.
  void *lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
  if (!lib)
    lib = dlopen("libcuda.so", RTLD_NOW | RTLD_LOCAL);
  if (!lib) {
    const char *why = dlerror();
    d.error = std::string("cannot load libcuda: ") + (why ? why : "unknown");
    return;
  }
  std::string &e = d.error;
  // Versioned entry points: the unsuffixed names are the legacy ABI.
  bool ok = bind(lib, d.Init, "cuInit", e) &&
            bind(lib, d.DriverGetVersion, "cuDriverGetVersion", e) &&
            bind(lib, d.DeviceGet, "cuDeviceGet", e) &&
            bind(lib, d.DeviceGetCount, "cuDeviceGetCount", e) &&
            bind(lib, d.DeviceGetName, "cuDeviceGetName", e) &&
            bind(lib, d.DeviceGetAttribute, "cuDeviceGetAttribute", e) &&
            bind(lib, d.DevicePrimaryCtxRetain, "cuDevicePrimaryCtxRetain", e) &&
            bind(lib, d.DevicePrimaryCtxRelease, "cuDevicePrimaryCtxRelease_v2",
                 e) &&
            bind(lib, d.CtxPushCurrent, "cuCtxPushCurrent_v2", e) &&
            bind(lib, d.CtxPopCurrent, "cuCtxPopCurrent_v2", e) &&
            bind(lib, d.CtxGetCurrent, "cuCtxGetCurrent", e) &&
            bind(lib, d.CtxSynchronize, "cuCtxSynchronize", e) &&
            bind(lib, d.CtxEnablePeerAccess, "cuCtxEnablePeerAccess", e) &&
            bind(lib, d.DeviceCanAccessPeer, "cuDeviceCanAccessPeer", e) &&
            bind(lib, d.StreamCreate, "cuStreamCreate", e) &&
            bind(lib, d.StreamCreateWithPriority, "cuStreamCreateWithPriority", e) &&
            bind(lib, d.CtxGetStreamPriorityRange, "cuCtxGetStreamPriorityRange", e) &&
            bind(lib, d.StreamDestroy, "cuStreamDestroy_v2", e) &&
            bind(lib, d.StreamSynchronize, "cuStreamSynchronize", e) &&
            bind(lib, d.StreamWaitEvent, "cuStreamWaitEvent", e) &&
            bind(lib, d.MemAlloc, "cuMemAlloc_v2", e) &&
            bind(lib, d.MemFree, "cuMemFree_v2", e) &&
            bind(lib, d.MemAllocHost, "cuMemAllocHost_v2", e) &&
            bind(lib, d.MemFreeHost, "cuMemFreeHost", e) &&
            bind(lib, d.MemHostAlloc, "cuMemHostAlloc", e) &&
            bind(lib, d.MemHostRegister, "cuMemHostRegister_v2", e) &&
            bind(lib, d.MemHostUnregister, "cuMemHostUnregister", e) &&
            bind(lib, d.MemcpyHtoDAsync, "cuMemcpyHtoDAsync_v2", e) &&
            bind(lib, d.MemcpyDtoHAsync, "cuMemcpyDtoHAsync_v2", e) &&
            bind(lib, d.MemcpyDtoDAsync, "cuMemcpyDtoDAsync_v2", e) &&
            bind(lib, d.Memcpy2DAsync, "cuMemcpy2DAsync_v2", e) &&
            bind(lib, d.MemcpyPeerAsync, "cuMemcpyPeerAsync", e) &&
            bind(lib, d.MemsetD8Async, "cuMemsetD8Async", e) &&
            bind(lib, d.MemsetD32Async, "cuMemsetD32Async", e) &&
            bind(lib, d.PointerGetAttribute, "cuPointerGetAttribute", e) &&
            bind(lib, d.MemGetAddressRange, "cuMemGetAddressRange_v2", e) &&
            bind(lib, d.IpcGetMemHandle, "cuIpcGetMemHandle", e) &&
            bind(lib, d.IpcOpenMemHandle, "cuIpcOpenMemHandle_v2", e) &&
            bind(lib, d.IpcCloseMemHandle, "cuIpcCloseMemHandle", e) &&
            bind(lib, d.ModuleLoadData, "cuModuleLoadData", e) &&
            bind(lib, d.ModuleUnload, "cuModuleUnload", e) &&
            bind(lib, d.ModuleGetFunction, "cuModuleGetFunction", e) &&
            bind(lib, d.ModuleGetGlobal, "cuModuleGetGlobal_v2", e) &&
            bind(lib, d.FuncSetAttribute, "cuFuncSetAttribute", e) &&
            bind(lib, d.LaunchKernel, "cuLaunchKernel", e) &&
            bind(lib, d.EventCreate, "cuEventCreate", e) &&
            bind(lib, d.EventDestroy, "cuEventDestroy_v2", e) &&
            bind(lib, d.EventRecord, "cuEventRecord", e) &&
            bind(lib, d.EventSynchronize, "cuEventSynchronize", e) &&
            bind(lib, d.EventElapsedTime, "cuEventElapsedTime", e) &&
            bind(lib, d.TensorMapEncodeTiled, "cuTensorMapEncodeTiled", e);
  if (!ok)
    return;
  // Optional: only used to make messages readable.
  d.GetErrorString =
      reinterpret_cast<decltype(d.GetErrorString)>(dlsym(lib, "cuGetErrorString"));
  d.LaunchKernelEx =
      reinterpret_cast<decltype(d.LaunchKernelEx)>(dlsym(lib, "cuLaunchKernelEx"));
  d.OccupancyMaxActiveClusters =
      reinterpret_cast<decltype(d.OccupancyMaxActiveClusters)>(
          dlsym(lib, "cuOccupancyMaxActiveClusters"));
  CUresult r = d.Init(0);
  if (r != CUDA_SUCCESS) {
    d.error = cuda_message("cuInit", r);
    return;
  }
  d.ok = true;
}

}  // namespace

const Driver &driver() {
  std::call_once(g_once, load);
  return g_driver;
}

std::string cuda_message(const char *call, CUresult result) {
  const char *msg = nullptr;
  const Driver &d = g_driver;
  if (d.GetErrorString && d.GetErrorString(result, &msg) == CUDA_SUCCESS && msg)
    return std::string(call) + " failed: " + msg;
  return std::string(call) + " failed: CUDA error " + std::to_string(result);
}

ContextGuard::ContextGuard(CUcontext ctx) {
  const Driver &d = driver();
  if (d.ok && ctx)
    pushed_ = d.CtxPushCurrent(ctx) == CUDA_SUCCESS;
}

ContextGuard::~ContextGuard() {
  if (pushed_) {
    CUcontext popped = nullptr;
    driver().CtxPopCurrent(&popped);
  }
}

}  // namespace hexir
