// kernel_lib.h -- per-GPU state and the launchers of the sm_100a kernels.
//
// One DeviceState per CUDA ordinal, created on first use and kept for the
// life of the process: the retained primary context (shared with any other
// library in the process, e.g. NCCL or PyTorch), the SM count, the loaded
// kernel modules keyed by image content, and the split-K workspace.
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "hexir_runtime/status.h"

namespace hexir {

struct KernelLib {
  CUmodule module = nullptr;
  CUfunction linear_tma = nullptr;      // 128-row tiles
  CUfunction linear_tma_m64 = nullptr;  // 64-row tiles
  CUfunction linear_tma_m16 = nullptr;  // 16-row tiles
  CUfunction linear_guarded = nullptr;
  CUfunction linear_tma_sk = nullptr;   // stream-K (absent in older images)
  CUfunction sk_fixup = nullptr;
  CUfunction splitk_reduce = nullptr;
  CUfunction relu = nullptr;
  CUfunction add = nullptr;
  // Activations (absent in images written before they existed): the
  // elementwise kernels by HEXIR_ACT_* code - 7 (the softmax slot stays
  // empty), then the four softmax launch shapes.
  CUfunction activation[8] = {};
  CUfunction softmax_warp = nullptr, softmax_b256 = nullptr,
             softmax_b512 = nullptr, softmax_wide = nullptr,
             softmax_bulk256 = nullptr, softmax_bulk512 = nullptr,
             softmax_bulk_s2k = nullptr, softmax_bulk_s4k = nullptr;
  // Long rows over thread-block clusters of 4-8 CTAs, by cluster size - 4
  // (all or none).
  CUfunction softmax_cluster[5] = {};
  CUfunction dmma_probe = nullptr;
  // The reference's generated schedule, a measurement baseline only
  // (absent in images written before it existed).
  CUfunction baseline_schedule = nullptr;
  CUfunction wait_probe = nullptr;
  CUdeviceptr error_word = 0;
};

struct DeviceState {
  int ordinal = -1;
  CUdevice device = 0;
  CUcontext context = nullptr;
  int sm_count = 0;
  std::string name;

  std::mutex mu;
  std::map<uint64_t, std::unique_ptr<KernelLib>> libs;  // by image hash
  KernelLib *embedded = nullptr;

  // split-K partial sums; reuse across streams is ordered by `ws_ready`.
  CUdeviceptr workspace = 0;
  size_t workspace_bytes = 0;
  CUevent ws_ready = nullptr;
};

// Per-ordinal state; nullptr (and *error set) if the GPU cannot be opened.
DeviceState *device_state(int ordinal, std::string *error);

// The kernel module for `image` on this device, loading it on first use.
// Returns nullptr with *error set if the image does not load or lacks the
// kernels of launch ABI version 1.
KernelLib *library_for_image(DeviceState *dev, const void *image, size_t size,
                             std::string *error);

// The library's own embedded image on this device.
KernelLib *embedded_library(DeviceState *dev, std::string *error);

// Matmul kernel variants (hexir_cuda_matmul_plan reports these numbers).
enum MatmulVariant {
  kTma128 = 1,   // hexir_linear_f64_tma, 128 x 128 x 32
  kGuarded = 2,  // hexir_linear_f64_guarded, 64 x 64 x 16, any shape
  kTma16 = 3,    // hexir_linear_f64_tma_m16, 16 x 128 x 32
  kTma64 = 4,    // hexir_linear_f64_tma_m64, 64 x 128 x 32
  kTma128Sk = 5, // hexir_linear_f64_tma_sk, 128 x 128 x 32, stream-K
};

struct MatmulPlan {
  int variant = 0;  // MatmulVariant
  uint32_t split_k = 1;
  uint32_t tiles_m = 0, tiles_n = 0, k_tiles = 0, k_tiles_per_split = 0;
  uint32_t bm = 0, bn = 0, bk = 0;
  // kTma128Sk: persistent grid, data-parallel tiles, k-tile units per CTA.
  uint32_t sk_grid = 0, sk_dp_tiles = 0, sk_units = 0;
  bool stream_k() const { return variant == kTma128Sk; }
};

// lda: row stride of a in elements (0 = k).  c_in: when non-null the sums
// start from c_in (no k split), see hexir_linear_args_t.  addend: when
// non-null, c = a . b + addend (before the relu), [m][n] like c.
MatmulPlan plan_matmul(const DeviceState *dev, const double *a, const double *b,
                       const double *c, uint32_t m, uint32_t n, uint32_t k,
                       uint32_t flags, uint32_t lda = 0,
                       const double *c_in = nullptr,
                       const double *addend = nullptr);

// Launchers.  The caller has made dev->context current.  All asynchronous.
hexir_status_t launch_matmul(DeviceState *dev, KernelLib *lib, const double *a,
                             const double *b, double *c, uint32_t m, uint32_t n,
                             uint32_t k, uint32_t flags, CUstream stream,
                             std::string *error, uint32_t lda = 0,
                             const double *c_in = nullptr,
                             const double *addend = nullptr);
hexir_status_t launch_relu(DeviceState *dev, KernelLib *lib, const double *x,
                           double *y, size_t n, CUstream stream,
                           std::string *error);
hexir_status_t launch_add(DeviceState *dev, KernelLib *lib, const double *a,
                          const double *b, double *c, size_t n, CUstream stream,
                          std::string *error);
// y = op(x) over rows x cols (HEXIR_ACT_* op; softmax along each row, the
// others elementwise over rows * cols).
hexir_status_t launch_activation(DeviceState *dev, KernelLib *lib, uint32_t op,
                                 const double *x, double *y, uint64_t rows,
                                 uint32_t cols, CUstream stream,
                                 std::string *error);

// Synchronise `stream` and collect (and clear) the device error word of
// every module loaded on this device.
hexir_status_t check_device(DeviceState *dev, CUstream stream,
                            std::string *error);

// Bounds 0 = b0 < b1 < ... = k1 of the k pieces in which a weight streamed
// from the host is used while the rest of it still arrives: 256 first, then
// each piece at most 256 + 0.7 x the k done so far (rounded to the 32-wide k
// tile), so a piece's upload (a column slice plus weight rows, ~2.25 ms per
// 1024 k at 8192 rows and columns over PCIe) ends before the previous
// pieces' compute (~3.9 ms per 1024 k) does.
std::vector<uint32_t> weight_stream_bounds(uint32_t k1);

void count_launch();
void set_last_error(const std::string &message);

// 64-bit FNV-1a over a byte range (image identity).
uint64_t hash_bytes(const void *data, size_t size);

// The CUBIN linked into this library (embedded_image.S).
const void *embedded_image_data();
size_t embedded_image_size();

}  // namespace hexir
