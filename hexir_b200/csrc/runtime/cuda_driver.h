// cuda_driver.h -- the slice of the CUDA driver API this runtime uses,
// resolved at run time from libcuda.so.1 with dlopen/dlsym.
//
// Like the reference backend (runtime/src/hal/cuda/cuda_device.c:25-117) the
// library links no CUDA library: a machine without a driver can still load
// it, run CPU programs, and get a clear error when it asks for a GPU.  Types
// and constants come from the toolkit's cuda.h at build time only.
#pragma once

#include <cuda.h>

#include <string>

namespace hexir {

struct Driver {
  bool ok = false;
  std::string error;  // why loading failed

  CUresult (*Init)(unsigned int) = nullptr;
  CUresult (*DriverGetVersion)(int *) = nullptr;
  CUresult (*DeviceGet)(CUdevice *, int) = nullptr;
  CUresult (*DeviceGetCount)(int *) = nullptr;
  CUresult (*DeviceGetName)(char *, int, CUdevice) = nullptr;
  CUresult (*DeviceGetAttribute)(int *, CUdevice_attribute, CUdevice) = nullptr;
  CUresult (*DevicePrimaryCtxRetain)(CUcontext *, CUdevice) = nullptr;
  CUresult (*DevicePrimaryCtxRelease)(CUdevice) = nullptr;
  CUresult (*CtxPushCurrent)(CUcontext) = nullptr;
  CUresult (*CtxPopCurrent)(CUcontext *) = nullptr;
  CUresult (*CtxGetCurrent)(CUcontext *) = nullptr;
  CUresult (*CtxSynchronize)(void) = nullptr;
  CUresult (*CtxEnablePeerAccess)(CUcontext, unsigned int) = nullptr;
  CUresult (*DeviceCanAccessPeer)(int *, CUdevice, CUdevice) = nullptr;
  CUresult (*StreamCreate)(CUstream *, unsigned int) = nullptr;
  CUresult (*StreamCreateWithPriority)(CUstream *, unsigned int, int) = nullptr;
  CUresult (*CtxGetStreamPriorityRange)(int *, int *) = nullptr;
  CUresult (*StreamDestroy)(CUstream) = nullptr;
  CUresult (*StreamSynchronize)(CUstream) = nullptr;
  CUresult (*StreamWaitEvent)(CUstream, CUevent, unsigned int) = nullptr;
  CUresult (*MemAlloc)(CUdeviceptr *, size_t) = nullptr;
  CUresult (*MemFree)(CUdeviceptr) = nullptr;
  CUresult (*MemAllocHost)(void **, size_t) = nullptr;
  CUresult (*MemFreeHost)(void *) = nullptr;
  CUresult (*MemHostAlloc)(void **, size_t, unsigned int) = nullptr;
  CUresult (*MemHostRegister)(void *, size_t, unsigned int) = nullptr;
  CUresult (*MemHostUnregister)(void *) = nullptr;
  CUresult (*MemcpyHtoDAsync)(CUdeviceptr, const void *, size_t, CUstream) =
      nullptr;
  CUresult (*MemcpyDtoHAsync)(void *, CUdeviceptr, size_t, CUstream) = nullptr;
  CUresult (*MemcpyDtoDAsync)(CUdeviceptr, CUdeviceptr, size_t, CUstream) =
      nullptr;
  CUresult (*Memcpy2DAsync)(const CUDA_MEMCPY2D *, CUstream) = nullptr;
  CUresult (*MemcpyPeerAsync)(CUdeviceptr, CUcontext, CUdeviceptr, CUcontext,
                              size_t, CUstream) = nullptr;
  CUresult (*MemsetD8Async)(CUdeviceptr, unsigned char, size_t, CUstream) =
      nullptr;
  CUresult (*MemsetD32Async)(CUdeviceptr, unsigned int, size_t, CUstream) =
      nullptr;
  CUresult (*PointerGetAttribute)(void *, CUpointer_attribute,
                                  CUdeviceptr) = nullptr;
  CUresult (*MemGetAddressRange)(CUdeviceptr *, size_t *, CUdeviceptr) = nullptr;
  CUresult (*IpcGetMemHandle)(CUipcMemHandle *, CUdeviceptr) = nullptr;
  CUresult (*IpcOpenMemHandle)(CUdeviceptr *, CUipcMemHandle, unsigned int) =
      nullptr;
  CUresult (*IpcCloseMemHandle)(CUdeviceptr) = nullptr;
  CUresult (*ModuleLoadData)(CUmodule *, const void *) = nullptr;
  CUresult (*ModuleUnload)(CUmodule) = nullptr;
  CUresult (*ModuleGetFunction)(CUfunction *, CUmodule, const char *) = nullptr;
  CUresult (*ModuleGetGlobal)(CUdeviceptr *, size_t *, CUmodule,
                              const char *) = nullptr;
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned,
                           unsigned, unsigned, unsigned, CUstream, void **,
                           void **) = nullptr;
  CUresult (*EventCreate)(CUevent *, unsigned int) = nullptr;
  CUresult (*EventDestroy)(CUevent) = nullptr;
  CUresult (*EventRecord)(CUevent, CUstream) = nullptr;
  CUresult (*EventSynchronize)(CUevent) = nullptr;
  CUresult (*EventElapsedTime)(float *, CUevent, CUevent) = nullptr;
  CUresult (*TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType,
                                   cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle,
                                   CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill) = nullptr;
  CUresult (*GetErrorString)(CUresult, const char **) = nullptr;
  // Optional (launches with a cluster shape): null on drivers without it.
  CUresult (*LaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **,
                             void **) = nullptr;
  CUresult (*OccupancyMaxActiveClusters)(int *, CUfunction,
                                         const CUlaunchConfig *) = nullptr;
};

// Loads libcuda once per process and calls cuInit(0).  Never null; check ok.
const Driver &driver();

// "<call> failed: <driver message>" for diagnostics.
std::string cuda_message(const char *call, CUresult result);

// Pushes `ctx` for the lifetime of the guard.
class ContextGuard {
 public:
  explicit ContextGuard(CUcontext ctx);
  ~ContextGuard();
  ContextGuard(const ContextGuard &) = delete;
  ContextGuard &operator=(const ContextGuard &) = delete;

 private:
  bool pushed_ = false;
};

}  // namespace hexir
