// matmul_noalloc.cu -- hexir_cuda_matmul_f64_noalloc: the f64 linear for
// callers that cannot allocate device memory (include/hexir_b200/kernels.h).
//
// Same contraction and flags as hexir_cuda_matmul_f64, computed by the
// bounds-checked DMMA kernel (hexir_linear_f64_guarded) and, when the k range
// is split, the split-order reduction.  The split-K partial sums live in
// `g_scratch` below, a fixed array in device memory that comes with this
// library's device code, instead of a workspace the library allocates.
//
// Set-up: the first call on each device makes that device current, asks the
// runtime for the array's device address (cudaGetSymbolAddress) and the SM
// count, and restores the previous device.  Later calls on that device only
// launch.  That first call should come before any stream capture.
//
// Sharing: every call on a device uses the same array and it keeps whatever
// the last call left there.  Nothing has to start at zero -- each launch
// writes every partial element it later reads -- but calls whose kernels
// overlap on the GPU (different streams, or threads racing on one device)
// overwrite each other's partial sums.  Serialise them.

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../kernels/launch_abi.h"
#include "hexir_b200/kernels.h"
#include "kernel_lib.h"

// The device code this path launches: its own copy of the guarded linear
// kernel and the split-K reduction (not of the TMA kernels, which it never
// launches).  Neither waits on anything but __syncthreads, so nothing sets
// the error word below and nothing reads it; it is defined only because the
// shared device helpers name one.  A variant of this path that launched a
// kernel with a bounded wait would have to read it back
// (cudaMemcpyFromSymbol) to report a timeout.
extern "C" {
__device__ unsigned int hexir_device_error_word = 0u;
}
#include "../kernels/linear_guarded_f64.cu"

// Split-K partial sums, HEXIR_NOALLOC_SCRATCH_BYTES of device memory on every
// GPU where this library's device code is loaded, held until the process
// exits.  In host code `g_scratch` only names the symbol (a host-side
// stand-in, not a device address): kernels get the pointer that
// cudaGetSymbolAddress returns for it.
static __device__ __align__(256)
    double g_scratch[HEXIR_NOALLOC_SCRATCH_BYTES / sizeof(double)];

namespace {

constexpr size_t kScratchDoubles = HEXIR_NOALLOC_SCRATCH_BYTES / sizeof(double);
constexpr int kMaxDevices = 64;

struct DeviceSetup {
  std::once_flag once;
  cudaError_t status = cudaErrorNotReady;
  double *scratch = nullptr;
  int sm_count = 0;
};

DeviceSetup g_setup[kMaxDevices];

void setup_device(int ordinal, DeviceSetup *s) {
  int previous = -1;
  cudaError_t e = cudaGetDevice(&previous);
  if (e == cudaSuccess)
    e = cudaSetDevice(ordinal);
  void *ptr = nullptr;
  if (e == cudaSuccess)
    e = cudaGetSymbolAddress(&ptr, g_scratch);
  int sms = 0;
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ordinal);
  if (previous >= 0)
    cudaSetDevice(previous);
  s->scratch = static_cast<double *>(ptr);
  s->sm_count = sms;
  s->status = e;
}

hexir_status_t fail(hexir_status_t status, const std::string &message) {
  hexir::set_last_error(message);
  return status;
}

unsigned ceil_div_u(uint64_t a, uint64_t b) {
  return static_cast<unsigned>((a + b - 1) / b);
}

}  // namespace

extern "C" hexir_status_t hexir_cuda_matmul_f64_noalloc(
    int ordinal, const double *a, const double *b, double *c, uint32_t m,
    uint32_t n, uint32_t k, uint32_t flags, void *stream) {
  if (ordinal < 0 || ordinal >= kMaxDevices)
    return fail(HEXIR_ERROR_INVALID_ARGUMENT, "no-alloc matmul: bad ordinal");
  if (m == 0 || n == 0)
    return HEXIR_OK;
  if (!a || !b || !c)
    return fail(HEXIR_ERROR_INVALID_ARGUMENT, "no-alloc matmul: null pointer");
  DeviceSetup *s = &g_setup[ordinal];
  std::call_once(s->once, setup_device, ordinal, s);
  if (s->status != cudaSuccess)
    return fail(HEXIR_ERROR_DEVICE,
                std::string("no-alloc matmul set-up on device ") +
                    std::to_string(ordinal) + ": " +
                    cudaGetErrorString(s->status));

  hexir::DeviceState shape_only;  // only sm_count is read by the planner
  shape_only.sm_count = s->sm_count;
  const hexir::MatmulPlan p = hexir::plan_matmul(
      &shape_only, a, b, c, m, n, k,
      (flags & ~HEXIR_MATMUL_FORCE_TMA) | HEXIR_MATMUL_FORCE_GUARDED);
  const uint64_t partial_doubles =
      p.split_k > 1 ? static_cast<uint64_t>(p.split_k) * m * n : 0;
  if (partial_doubles > kScratchDoubles)
    return fail(HEXIR_ERROR_INVALID_ARGUMENT,
                "no-alloc matmul: " + std::to_string(m) + "x" +
                    std::to_string(n) + " split " + std::to_string(p.split_k) +
                    " ways needs " + std::to_string(partial_doubles * 8) +
                    " bytes of scratch; the fixed scratch holds " +
                    std::to_string(HEXIR_NOALLOC_SCRATCH_BYTES) + " bytes");

  int previous = -1;
  cudaGetDevice(&previous);
  if (previous != ordinal)
    cudaSetDevice(ordinal);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  hexir_linear_args_t args = {};
  args.a = a;
  args.b = b;
  args.c = p.split_k > 1 ? s->scratch : c;
  args.m = m;
  args.n = n;
  args.k = k;
  args.epilogue = (flags & HEXIR_MATMUL_RELU) ? HEXIR_EPILOGUE_RELU : 0u;
  args.tiles_m = p.tiles_m;
  args.tiles_n = p.tiles_n;
  args.group_m = p.tiles_m < 8 ? p.tiles_m : 8;
  args.k_tiles = p.k_tiles;
  args.split_k = p.split_k;
  args.k_tiles_per_split = p.k_tiles_per_split;
  args.timeout_ns = 4000000000ull;  // unused: the guarded kernel has no waits

  cudaError_t e = cudaSuccess;
  if (k == 0) {
    e = cudaMemsetAsync(c, 0, static_cast<size_t>(m) * n * sizeof(double), st);
  } else {
    hexir_linear_f64_guarded<<<dim3(p.tiles_m * p.tiles_n, p.split_k),
                               HEXIR_LINEAR_G_THREADS,
                               HEXIR_LINEAR_G_SMEM_BYTES, st>>>(args);
    e = cudaGetLastError();
    if (e == cudaSuccess)
      hexir::count_launch();
    if (e == cudaSuccess && p.split_k > 1) {
      hexir_reduce_args_t red;
      red.partials = s->scratch;
      red.c = c;
      red.count = static_cast<uint64_t>(m) * n;
      red.split = p.split_k;
      red.epilogue = args.epilogue;
      const unsigned want = ceil_div_u(red.count, 256);
      const unsigned cap = static_cast<unsigned>(s->sm_count > 0 ? s->sm_count : 1) * 8;
      hexir_linear_f64_splitk_reduce<<<want < cap ? (want ? want : 1) : cap, 256,
                                       0, st>>>(red);
      e = cudaGetLastError();
      if (e == cudaSuccess)
        hexir::count_launch();
    }
  }
  if (previous >= 0 && previous != ordinal)
    cudaSetDevice(previous);
  if (e != cudaSuccess)
    return fail(HEXIR_ERROR_DEVICE, std::string("no-alloc matmul launch: ") +
                                        cudaGetErrorString(e));
  return HEXIR_OK;
}
