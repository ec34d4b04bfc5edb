// kernel_lib.cc -- per-GPU state, kernel module cache, launch planning and the
// kernel-level C ABI (include/hexir_b200/kernels.h).

#include "kernel_lib.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>

#include "../kernels/launch_abi.h"
#include "cuda_driver.h"
#include "fault.h"
#include "hexir_b200/kernels.h"

extern "C" {
extern const unsigned char hexir_embedded_cubin_begin[];
extern const unsigned char hexir_embedded_cubin_end[];
}

namespace hexir {

namespace {

std::mutex g_devices_mu;
std::map<int, std::unique_ptr<DeviceState>> g_devices;
std::atomic<uint64_t> g_launches{0};
thread_local std::string g_last_error;

// Every pipeline wait in the kernels gives up after this much wall time.
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;

bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

uint32_t ceil_div(uint64_t a, uint64_t b) {
  return static_cast<uint32_t>((a + b - 1) / b);
}

hexir_status_t fail(std::string *error, std::string message,
                    hexir_status_t status = HEXIR_ERROR_DEVICE) {
  if (error)
    *error = std::move(message);
  return status;
}

// Workspace for split-K partials: grown on demand, never shrunk.  Growing
// frees the old block only after the context is idle.
hexir_status_t ensure_workspace(DeviceState *dev, size_t bytes,
                                std::string *error) {
  const Driver &d = driver();
  if (dev->workspace_bytes >= bytes)
    return HEXIR_OK;
  if (dev->workspace) {
    d.CtxSynchronize();
    d.MemFree(dev->workspace);
    dev->workspace = 0;
    dev->workspace_bytes = 0;
  }
  CUresult r = fault_hit(FaultSite::Alloc) ? CUDA_ERROR_OUT_OF_MEMORY
                                           : d.MemAlloc(&dev->workspace, bytes);
  if (r != CUDA_SUCCESS)
    return fail(error, cuda_message("cuMemAlloc(split-K workspace)", r),
                HEXIR_ERROR_OUT_OF_MEMORY);
  dev->workspace_bytes = bytes;
  return HEXIR_OK;
}

hexir_status_t launch(CUfunction fn, unsigned gx, unsigned gy, unsigned bx,
                      unsigned smem, CUstream stream, void **params,
                      const char *what, std::string *error) {
  if (fault_hit(FaultSite::Launch))
    return fail(error, std::string(what) + ": injected fault (HEXIR_FAULT)");
  CUresult r =
      driver().LaunchKernel(fn, gx, gy, 1, bx, 1, 1, smem, stream, params, nullptr);
  if (r != CUDA_SUCCESS)
    return fail(error, cuda_message(what, r));
  count_launch();
  return HEXIR_OK;
}

// A launch that depends on the kernel queued before it on `stream` only
// through memory: with programmatic stream serialization its CTAs may be
// placed while that kernel's last CTAs run, and the kernel itself waits
// (griddepcontrol.wait) for that kernel's completion before reading.  Hides
// the launch gap between a GEMM and its split-K reduction or stream-K
// fix-up.  A plain launch where the driver has no cuLaunchKernelEx.
hexir_status_t launch_after(CUfunction fn, unsigned gx, unsigned gy,
                            unsigned bx, CUstream stream, void **params,
                            const char *what, std::string *error) {
  const Driver &d = driver();
  if (!d.LaunchKernelEx)
    return launch(fn, gx, gy, bx, 0, stream, params, what, error);
  if (fault_hit(FaultSite::Launch))
    return fail(error, std::string(what) + ": injected fault (HEXIR_FAULT)");
  CUlaunchAttribute attr;
  std::memset(&attr, 0, sizeof(attr));
  attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr.value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDimX = gx;
  cfg.gridDimY = gy;
  cfg.gridDimZ = 1;
  cfg.blockDimX = bx;
  cfg.blockDimY = 1;
  cfg.blockDimZ = 1;
  cfg.hStream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const CUresult r = d.LaunchKernelEx(&cfg, fn, params, nullptr);
  if (r != CUDA_SUCCESS)
    return fail(error, cuda_message(what, r));
  count_launch();
  return HEXIR_OK;
}

// The launch configuration of `gx` CTAs in clusters of `cluster` along x.
struct ClusterLaunch {
  CUlaunchAttribute attr;
  CUlaunchConfig cfg;
  ClusterLaunch(unsigned gx, unsigned cluster, unsigned bx, unsigned smem,
                CUstream stream) {
    std::memset(&attr, 0, sizeof(attr));
    attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr.value.clusterDim.x = cluster;
    attr.value.clusterDim.y = 1;
    attr.value.clusterDim.z = 1;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDimX = gx;
    cfg.gridDimY = 1;
    cfg.gridDimZ = 1;
    cfg.blockDimX = bx;
    cfg.blockDimY = 1;
    cfg.blockDimZ = 1;
    cfg.sharedMemBytes = smem;
    cfg.hStream = stream;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
  }
};

// How many clusters of this shape can be resident at once: clusters are
// placed inside a GPC, so fewer fit than SMs / cluster size suggests.  0 if
// the driver cannot say.
unsigned max_active_clusters(CUfunction fn, unsigned cluster, unsigned bx,
                             unsigned smem) {
  const Driver &d = driver();
  if (!d.OccupancyMaxActiveClusters)
    return 0;
  ClusterLaunch l(cluster, cluster, bx, smem, nullptr);
  int n = 0;
  return d.OccupancyMaxActiveClusters(&n, fn, &l.cfg) == CUDA_SUCCESS && n > 0
             ? static_cast<unsigned>(n)
             : 0u;
}

// A launch with a cluster shape of `cluster` CTAs along x.
hexir_status_t launch_cluster(CUfunction fn, unsigned gx, unsigned cluster,
                              unsigned bx, unsigned smem, CUstream stream,
                              void **params, const char *what,
                              std::string *error) {
  if (fault_hit(FaultSite::Launch))
    return fail(error, std::string(what) + ": injected fault (HEXIR_FAULT)");
  const Driver &d = driver();
  if (!d.LaunchKernelEx)
    return fail(error, std::string(what) + ": the driver has no cuLaunchKernelEx");
  ClusterLaunch l(gx, cluster, bx, smem, stream);
  const CUresult r = d.LaunchKernelEx(&l.cfg, fn, params, nullptr);
  if (r != CUDA_SUCCESS)
    return fail(error, cuda_message(what, r));
  count_launch();
  return HEXIR_OK;
}

unsigned stream_grid(const DeviceState *dev, uint64_t pairs) {
  // Four 16-byte vectors per thread per pass, 256 threads per CTA; at most
  // 8 CTAs per SM, the rest by grid stride.
  const uint64_t want = (pairs + 1023) / 1024;
  const uint64_t cap = static_cast<uint64_t>(std::max(dev->sm_count, 1)) * 8;
  return static_cast<unsigned>(std::max<uint64_t>(1, std::min(want, cap)));
}

}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

std::vector<uint32_t> weight_stream_bounds(uint32_t k1) {
  std::vector<uint32_t> b{0};
  const uint32_t first = std::min<uint32_t>(256, k1);
  uint32_t done = 0;
  while (done < k1) {
    uint32_t len = done == 0 ? first : (first + done * 7 / 10) / 32 * 32;
    len = std::max<uint32_t>(len, 32);
    if (done + len >= k1 || k1 - (done + len) < len / 2)
      len = k1 - done;
    done += len;
    b.push_back(done);
  }
  return b;
}

void set_last_error(const std::string &message) { g_last_error = message; }

uint64_t hash_bytes(const void *data, size_t size) {
  // FNV-1a over 8-byte words, then the tail bytes.
  const unsigned char *p = static_cast<const unsigned char *>(data);
  uint64_t h = 1469598103934665603ull;
  size_t i = 0;
  for (; i + 8 <= size; i += 8) {
    uint64_t w;
    std::memcpy(&w, p + i, 8);
    h ^= w;
    h *= 1099511628211ull;
  }
  for (; i < size; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h ^ size;
}

const void *embedded_image_data() { return hexir_embedded_cubin_begin; }
size_t embedded_image_size() {
  return static_cast<size_t>(hexir_embedded_cubin_end - hexir_embedded_cubin_begin);
}

DeviceState *device_state(int ordinal, std::string *error) {
  const Driver &d = driver();
  if (!d.ok) {
    if (error)
      *error = d.error;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_devices_mu);
  auto it = g_devices.find(ordinal);
  if (it != g_devices.end())
    return it->second.get();

  int count = 0;
  CUresult r = d.DeviceGetCount(&count);
  if (r != CUDA_SUCCESS) {
    fail(error, cuda_message("cuDeviceGetCount", r));
    return nullptr;
  }
  if (ordinal < 0 || ordinal >= count) {
    fail(error, "no CUDA device " + std::to_string(ordinal) + " (" +
                    std::to_string(count) + " visible)");
    return nullptr;
  }
  auto dev = std::make_unique<DeviceState>();
  dev->ordinal = ordinal;
  r = d.DeviceGet(&dev->device, ordinal);
  if (r == CUDA_SUCCESS)
    r = d.DevicePrimaryCtxRetain(&dev->context, dev->device);
  if (r != CUDA_SUCCESS) {
    fail(error, "cannot open CUDA device " + std::to_string(ordinal) + ": " +
                    cuda_message("cuDevicePrimaryCtxRetain", r));
    return nullptr;
  }
  d.DeviceGetAttribute(&dev->sm_count, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT,
                       dev->device);
  char name[128] = {0};
  if (d.DeviceGetName(name, sizeof(name) - 1, dev->device) == CUDA_SUCCESS)
    dev->name = name;
  {
    ContextGuard guard(dev->context);
    d.EventCreate(&dev->ws_ready, CU_EVENT_DISABLE_TIMING);
  }
  DeviceState *raw = dev.get();
  g_devices[ordinal] = std::move(dev);
  return raw;
}

KernelLib *library_for_image(DeviceState *dev, const void *image, size_t size,
                             std::string *error) {
  // Modules written by this library carry its own image: recognise it by a
  // memcmp (tens of microseconds) instead of hashing it on every execute.
  if (image != embedded_image_data() && size == embedded_image_size() &&
      std::memcmp(image, embedded_image_data(), size) == 0)
    return embedded_library(dev, error);
  const Driver &d = driver();
  const uint64_t key = hash_bytes(image, size);
  std::lock_guard<std::mutex> lock(dev->mu);
  auto it = dev->libs.find(key);
  if (it != dev->libs.end())
    return it->second.get();

  ContextGuard guard(dev->context);
  auto lib = std::make_unique<KernelLib>();
  CUresult r = d.ModuleLoadData(&lib->module, image);
  if (r != CUDA_SUCCESS) {
    int major = 0, minor = 0;
    d.DeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR,
                         dev->device);
    d.DeviceGetAttribute(&minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR,
                         dev->device);
    fail(error, cuda_message("cuModuleLoadData", r) +
                    " (the kernels are built for sm_100a; device " +
                    std::to_string(dev->ordinal) + " is sm_" +
                    std::to_string(major) + std::to_string(minor) + ")");
    return nullptr;
  }
  struct Need {
    CUfunction *slot;
    const char *name;
  } needs[] = {
      {&lib->linear_tma, "hexir_linear_f64_tma"},
      {&lib->linear_tma_m64, "hexir_linear_f64_tma_m64"},
      {&lib->linear_tma_m16, "hexir_linear_f64_tma_m16"},
      {&lib->linear_guarded, "hexir_linear_f64_guarded"},
      {&lib->splitk_reduce, "hexir_linear_f64_splitk_reduce"},
      {&lib->relu, "hexir_relu_f64"},
      {&lib->add, "hexir_add_f64"},
      {&lib->dmma_probe, "hexir_dmma_peak_probe"},
      {&lib->wait_probe, "hexir_wait_timeout_probe"},
  };
  CUfunction marker = nullptr;
  if (d.ModuleGetFunction(&marker, lib->module, "hexir_b200_abi_v1") !=
      CUDA_SUCCESS) {
    d.ModuleUnload(lib->module);
    fail(error, "device image is not a hexir-b200 kernel library (launch ABI "
                "version 1)");
    return nullptr;
  }
  for (const Need &need : needs) {
    r = d.ModuleGetFunction(need.slot, lib->module, need.name);
    if (r != CUDA_SUCCESS) {
      d.ModuleUnload(lib->module);
      fail(error, std::string("kernel library image lacks ") + need.name);
      return nullptr;
    }
  }
  // Optional: the baseline restating the reference's generated schedule.
  if (d.ModuleGetFunction(&lib->baseline_schedule, lib->module,
                          "hexir_baseline_reference_schedule_f64") !=
      CUDA_SUCCESS)
    lib->baseline_schedule = nullptr;
  // Optional: images written before the stream-K kernels existed lack them.
  if (d.ModuleGetFunction(&lib->linear_tma_sk, lib->module,
                          "hexir_linear_f64_tma_sk") != CUDA_SUCCESS ||
      d.ModuleGetFunction(&lib->sk_fixup, lib->module,
                          "hexir_linear_f64_sk_fixup") != CUDA_SUCCESS)
    lib->linear_tma_sk = lib->sk_fixup = nullptr;
  // Optional: the activation kernels, all or none.
  {
    struct Opt {
      CUfunction *slot;
      const char *name;
    } acts[] = {
        {&lib->activation[HEXIR_ACT_LEAKY_RELU - 7], "hexir_leaky_relu_f64"},
        {&lib->activation[HEXIR_ACT_ELU - 7], "hexir_elu_f64"},
        {&lib->activation[HEXIR_ACT_SIGMOID - 7], "hexir_sigmoid_f64"},
        {&lib->activation[HEXIR_ACT_TANH - 7], "hexir_tanh_f64"},
        {&lib->activation[HEXIR_ACT_GELU - 7], "hexir_gelu_f64"},
        {&lib->activation[HEXIR_ACT_SWISH - 7], "hexir_swish_f64"},
        {&lib->activation[HEXIR_ACT_MISH - 7], "hexir_mish_f64"},
        {&lib->softmax_warp, "hexir_softmax_warp_f64"},
        {&lib->softmax_b256, "hexir_softmax_b256_f64"},
        {&lib->softmax_b512, "hexir_softmax_b512_f64"},
        {&lib->softmax_wide, "hexir_softmax_wide_f64"},
        {&lib->softmax_bulk256, "hexir_softmax_bulk256_f64"},
        {&lib->softmax_bulk512, "hexir_softmax_bulk512_f64"},
    };
    bool all = true;
    for (const Opt &o : acts)
      all = all && d.ModuleGetFunction(o.slot, lib->module, o.name) == CUDA_SUCCESS;
    if (!all) {
      for (const Opt &o : acts)
        *o.slot = nullptr;
    }
  }
  // Optional: the short-row softmax blocks (rows in at most 16 / 32 KiB of
  // shared memory, under the default dynamic limit), both or neither.
  if (lib->softmax_bulk256 &&
      (d.ModuleGetFunction(&lib->softmax_bulk_s2k, lib->module,
                           "hexir_softmax_bulk_s2k_f64") != CUDA_SUCCESS ||
       d.ModuleGetFunction(&lib->softmax_bulk_s4k, lib->module,
                           "hexir_softmax_bulk_s4k_f64") != CUDA_SUCCESS))
    lib->softmax_bulk_s2k = lib->softmax_bulk_s4k = nullptr;
  // Optional: the cluster softmax for long rows, each CTA holding up to
  // 8192 columns (64 KiB of shared memory).
  {
    const char *names[5] = {
        "hexir_softmax_cluster4_f64", "hexir_softmax_cluster5_f64",
        "hexir_softmax_cluster6_f64", "hexir_softmax_cluster7_f64",
        "hexir_softmax_cluster8_f64"};
    bool all = lib->softmax_bulk256 != nullptr;
    for (int i = 0; i < 5 && all; ++i)
      all = d.ModuleGetFunction(&lib->softmax_cluster[i], lib->module,
                                names[i]) == CUDA_SUCCESS &&
            d.FuncSetAttribute(lib->softmax_cluster[i],
                               CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                               HEXIR_SOFTMAX_B256_COLS * 8) == CUDA_SUCCESS;
    if (!all)
      for (CUfunction &f : lib->softmax_cluster)
        f = nullptr;
  }
  size_t word_bytes = 0;
  r = d.ModuleGetGlobal(&lib->error_word, &word_bytes, lib->module,
                        "hexir_device_error_word");
  if (r == CUDA_SUCCESS)
    r = d.FuncSetAttribute(lib->linear_tma,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_LINEAR_SMEM_BYTES);
  if (r == CUDA_SUCCESS)
    r = d.FuncSetAttribute(lib->linear_tma_m64,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_LINEAR_M64_SMEM_BYTES);
  if (r == CUDA_SUCCESS)
    r = d.FuncSetAttribute(lib->linear_tma_m16,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_LINEAR_M16_SMEM_BYTES);
  if (r == CUDA_SUCCESS)
    r = d.FuncSetAttribute(lib->linear_guarded,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_LINEAR_G_SMEM_BYTES);
  if (r == CUDA_SUCCESS && lib->linear_tma_sk)
    r = d.FuncSetAttribute(lib->linear_tma_sk,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_LINEAR_SMEM_BYTES);
  // The bulk softmax blocks hold one row of up to 8192 / 16384 f64.
  if (r == CUDA_SUCCESS && lib->softmax_bulk256)
    r = d.FuncSetAttribute(lib->softmax_bulk256,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_SOFTMAX_B256_COLS * 8);
  if (r == CUDA_SUCCESS && lib->softmax_bulk512)
    r = d.FuncSetAttribute(lib->softmax_bulk512,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                           HEXIR_SOFTMAX_B512_COLS * 8);
  if (r != CUDA_SUCCESS) {
    d.ModuleUnload(lib->module);
    fail(error, cuda_message("kernel library setup", r));
    return nullptr;
  }
  KernelLib *raw = lib.get();
  dev->libs[key] = std::move(lib);
  return raw;
}

KernelLib *embedded_library(DeviceState *dev, std::string *error) {
  if (dev->embedded)
    return dev->embedded;
  KernelLib *lib = library_for_image(dev, embedded_image_data(),
                                     embedded_image_size(), error);
  if (lib) {
    std::lock_guard<std::mutex> lock(dev->mu);
    dev->embedded = lib;
  }
  return lib;
}

MatmulPlan plan_matmul(const DeviceState *dev, const double *a, const double *b,
                       const double *c, uint32_t m, uint32_t n, uint32_t k,
                       uint32_t flags, uint32_t lda, const double *c_in,
                       const double *addend) {
  MatmulPlan p;
  if (lda == 0)
    lda = k;
  // TMA needs 16-byte aligned bases and row strides (k, lda, n even); the
  // epilogue's paired accesses need the same of c, c_in and the addend.
  const bool tma_ok = (k % 2 == 0) && (lda % 2 == 0) && (n % 2 == 0) &&
                      aligned16(a) && aligned16(b) && aligned16(c) &&
                      aligned16(c_in) && aligned16(addend);
  if ((flags & HEXIR_MATMUL_FORCE_GUARDED) || !tma_ok) {
    p.variant = kGuarded;
    p.bm = HEXIR_LINEAR_G_BM;
    p.bn = HEXIR_LINEAR_G_BN;
    p.bk = HEXIR_LINEAR_G_BK;
  } else {
    // Row tile to the row count: a skinny a streams the weight once through
    // 16-row tiles instead of multiplying 112 rows of zero fill.
    p.variant = m <= 16 ? kTma16 : (m <= 64 ? kTma64 : kTma128);
    p.bm = p.variant == kTma16 ? 16u : (p.variant == kTma64 ? 64u : 128u);
    p.bn = HEXIR_LINEAR_BN;
    p.bk = HEXIR_LINEAR_BK;
  }
  p.tiles_m = ceil_div(m, p.bm);
  p.tiles_n = ceil_div(n, p.bn);
  p.k_tiles = ceil_div(k, p.bk);
  const uint64_t tiles = static_cast<uint64_t>(p.tiles_m) * p.tiles_n;
  uint32_t split = c_in ? 1u : (flags >> 16) & 0xFFu;
  const uint64_t sms = dev ? static_cast<uint64_t>(std::max(dev->sm_count, 1)) : 148;
  // CTAs resident per SM: one for the 128- and 64-row TMA tiles (192 KiB of
  // shared memory), two for the 16-row tile (109 KiB), three for the guarded
  // kernel (register bound).
  const uint64_t slots =
      sms * (p.variant == kGuarded ? 3 : (p.variant == kTma16 ? 2 : 1));
  if (split == 0) {
    // Pick the k split that minimises the modelled time, in units of one
    // CTA's k-tile: waves of CTAs, each running its share of k-tiles plus a
    // pipeline fill of 0.6 k-tile, plus the split-K reduction's HBM traffic
    // ((split + 1) * m * n * 8 bytes at ~6.4 TB/s).  Pieces keep >= 4
    // k-tiles so the pipeline still streams.  The constants were fitted to
    // B200 measurements of 1024^3, 2048^3, 8192x1024x4096 and m = 1..128
    // rows against 8192^2 (within ~5 %).
    // Seconds per k-tile per CTA: DMMA time of the tile at 64 FMA/clk and
    // ~1.9 GHz (the 16-row tile is bound instead by its 36 KiB weight stream,
    // two CTAs sharing an SM's ~43 GB/s share of HBM).
    double t_ktile = 4.3e-6;
    if (p.variant == kTma64)
      t_ktile = 2.15e-6;
    else if (p.variant == kTma16)
      t_ktile = 1.7e-6;
    else if (p.variant == kGuarded)
      t_ktile = 1.6e-6;
    split = 1;
    if (tiles < 4 * slots) {
      const uint32_t max_split =
          std::min<uint32_t>(64, std::max<uint32_t>(1, p.k_tiles / 4));
      double best = 0.0;
      for (uint32_t s = 1; s <= max_split; ++s) {
        const uint64_t ctas = tiles * s;
        const uint64_t waves = (ctas + slots - 1) / slots;
        const double per_cta = std::ceil(static_cast<double>(p.k_tiles) / s) + 0.6;
        double t = static_cast<double>(waves) * per_cta;
        if (s > 1)
          t += (s + 1.0) * m * n * 8.0 / 6.4e12 / t_ktile;
        if (s == 1 || t < best * 0.99) {  // a larger split must win by 1 %
          best = t;
          split = s;
        }
      }
    }
  }
  split = std::max<uint32_t>(1, std::min(split, std::max<uint32_t>(p.k_tiles, 1)));
  p.k_tiles_per_split = std::max<uint32_t>(1, ceil_div(p.k_tiles, split));
  // No empty pieces.
  p.split_k = std::max<uint32_t>(1, ceil_div(std::max<uint32_t>(p.k_tiles, 1),
                                             p.k_tiles_per_split));

  // Stream-K for the 128-row tiles: whole waves of tiles stay
  // data-parallel except the last one or two, whose k-tile units are dealt
  // out evenly over one CTA per SM (runs of >= 4 units); a fix-up kernel
  // sums the tiles split over CTAs.  (Keeping every whole wave
  // data-parallel measured equal or slower: 512x8192x8192 34.9 against
  // 35.3 TFLOP/s, 3072^3 34.4 against 34.6.)  Chosen by itself wherever
  // the wave model above splits k: measured on B200 it beats the split-K
  // schedule at every such shape tried (1024^3 29.8 against 26.2 TFLOP/s,
  // 2048^3 33.1 against 31.5, 256x2048x8192 33.6 against 31.9,
  // 512x8192x8192 35.6 against 34.3).  On request (FORCE_STREAM_K)
  // elsewhere, where it does not win (8192^3 34.9 against 35.2).  Never with
  // an explicit split, continued sums (c_in) or NO_STREAM_K: callers that
  // compute a matmul's rows in pieces pass that flag, since stream-K's
  // partial sums follow the whole tile set and row pieces could not
  // reproduce them.
  const bool explicit_split = ((flags >> 16) & 0xFFu) != 0;
  const bool want_sk = (flags & HEXIR_MATMUL_FORCE_STREAM_K) || p.split_k > 1;
  if (want_sk && p.variant == kTma128 && !c_in && !explicit_split &&
      !(flags & HEXIR_MATMUL_NO_STREAM_K) && sms > 0) {
    const uint64_t g = sms;
    const uint64_t dp_tiles = tiles >= 2 * g ? (tiles / g - 1) * g : 0;
    const uint64_t units = ((tiles - dp_tiles) * p.k_tiles + g - 1) / g;
    if (units >= 4) {
      p.variant = kTma128Sk;
      p.split_k = 1;
      p.k_tiles_per_split = p.k_tiles;
      p.sk_grid = static_cast<uint32_t>(g);
      p.sk_dp_tiles = static_cast<uint32_t>(dp_tiles);
      p.sk_units = static_cast<uint32_t>(units);
    }
  }
  return p;
}

hexir_status_t launch_matmul(DeviceState *dev, KernelLib *lib, const double *a,
                             const double *b, double *c, uint32_t m, uint32_t n,
                             uint32_t k, uint32_t flags, CUstream stream,
                             std::string *error, uint32_t lda,
                             const double *c_in, const double *addend) {
  const Driver &d = driver();
  if (m == 0 || n == 0)
    return HEXIR_OK;
  if (!a || !b || !c)
    return fail(error, "matmul: null pointer", HEXIR_ERROR_INVALID_ARGUMENT);
  if (lda == 0)
    lda = k;
  if (lda < k)
    return fail(error, "matmul: lda is smaller than k",
                HEXIR_ERROR_INVALID_ARGUMENT);
  if (c_in && (flags & 0xFF0000u) && ((flags >> 16) & 0xFFu) != 1)
    return fail(error, "matmul: a continued sum cannot be split over k",
                HEXIR_ERROR_INVALID_ARGUMENT);
  if ((flags & HEXIR_MATMUL_FORCE_TMA) &&
      plan_matmul(dev, a, b, c, m, n, k, flags & ~HEXIR_MATMUL_FORCE_TMA, lda,
                  c_in, addend)
              .variant == kGuarded)
    return fail(error,
                "matmul: the TMA kernel needs even k, lda and n and 16-byte "
                "aligned pointers",
                HEXIR_ERROR_INVALID_ARGUMENT);
  const size_t out_bytes = static_cast<size_t>(m) * n * sizeof(double);
  if (k == 0 && addend) {
    // An empty sum plus the addend: the add (and relu) kernels' arithmetic.
    const double *base = c_in;
    if (!base) {
      CUresult r = d.MemsetD8Async(reinterpret_cast<CUdeviceptr>(c), 0,
                                   out_bytes, stream);
      if (r != CUDA_SUCCESS)
        return fail(error, cuda_message("empty matmul", r));
      base = c;
    }
    hexir_status_t st = launch_add(dev, lib, base, addend, c,
                                   static_cast<size_t>(m) * n, stream, error);
    if (st != HEXIR_OK || !(flags & HEXIR_MATMUL_RELU))
      return st;
    return launch_relu(dev, lib, c, c, static_cast<size_t>(m) * n, stream, error);
  }
  if (k == 0) {
    // An empty sum is 0 (or c_in) and relu(0) = 0.
    CUresult r;
    if (!c_in) {
      r = d.MemsetD8Async(reinterpret_cast<CUdeviceptr>(c), 0, out_bytes, stream);
    } else if (!(flags & HEXIR_MATMUL_RELU)) {
      r = c_in == c ? CUDA_SUCCESS
                    : d.MemcpyDtoDAsync(reinterpret_cast<CUdeviceptr>(c),
                                        reinterpret_cast<CUdeviceptr>(c_in),
                                        out_bytes, stream);
    } else {
      return launch_relu(dev, lib, c_in, c, static_cast<size_t>(m) * n, stream,
                         error);
    }
    return r == CUDA_SUCCESS ? HEXIR_OK
                             : fail(error, cuda_message("empty matmul", r));
  }
  MatmulPlan p = plan_matmul(dev, a, b, c, m, n, k, flags, lda, c_in, addend);
  if (p.stream_k() && !lib->linear_tma_sk)  // an image without stream-K
    p = plan_matmul(dev, a, b, c, m, n, k, flags | HEXIR_MATMUL_NO_STREAM_K, lda,
                    c_in, addend);

  hexir_linear_args_t args;
  std::memset(&args, 0, sizeof(args));
  args.a = a;
  args.b = b;
  args.c = c;
  args.m = m;
  args.n = n;
  args.k = k;
  args.epilogue = ((flags & HEXIR_MATMUL_RELU) ? HEXIR_EPILOGUE_RELU : 0u) |
                  ((flags & HEXIR_MATMUL_REMOTE_OUTPUT) ? HEXIR_EPILOGUE_SYSTEM_FENCE
                                                        : 0u);
  args.tiles_m = p.tiles_m;
  args.tiles_n = p.tiles_n;
  args.group_m = std::min<uint32_t>(8, p.tiles_m);
  args.k_tiles = p.k_tiles;
  args.split_k = p.split_k;
  args.k_tiles_per_split = p.k_tiles_per_split;
  args.error = reinterpret_cast<unsigned int *>(lib->error_word);
  args.timeout_ns = kWaitTimeoutNs;
  args.c_in = c_in;
  args.lda = lda;
  args.addend = addend;
  if (addend)
    args.epilogue |= HEXIR_EPILOGUE_ADD;
  // 256-bit epilogue accesses where every row of c (the split-K partials
  // included), c_in and the addend starts on a 32-byte boundary.
  const bool rows32 = n % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(c) & 31u) == 0 &&
                      (reinterpret_cast<uintptr_t>(c_in) & 31u) == 0 &&
                      (reinterpret_cast<uintptr_t>(addend) & 31u) == 0;

  std::unique_lock<std::mutex> ws_lock(dev->mu, std::defer_lock);
  if (p.stream_k()) {
    // Partial tiles of the k units split over CTAs: two slots per CTA.
    ws_lock.lock();
    hexir_status_t s = ensure_workspace(
        dev, static_cast<size_t>(2) * p.sk_grid * HEXIR_LINEAR_BM *
                 HEXIR_LINEAR_BN * sizeof(double),
        error);
    if (s != HEXIR_OK)
      return s;
    d.StreamWaitEvent(stream, dev->ws_ready, 0);
    args.sk_partials = reinterpret_cast<double *>(dev->workspace);
    args.sk_dp_tiles = p.sk_dp_tiles;
    args.sk_units = p.sk_units;
  }
  if (p.split_k > 1) {
    ws_lock.lock();
    hexir_status_t s = ensure_workspace(
        dev, static_cast<size_t>(p.split_k) * out_bytes, error);
    if (s != HEXIR_OK)
      return s;
    // The previous user of the workspace may be another stream.
    d.StreamWaitEvent(stream, dev->ws_ready, 0);
    args.c = reinterpret_cast<double *>(dev->workspace);
  }
  if (rows32 && (reinterpret_cast<uintptr_t>(args.c) & 31u) == 0)
    args.epilogue |= HEXIR_EPILOGUE_VEC4;
  // A final output (not split-K partials, which the reduce reads back):
  // evict-first stores, so c does not displace a's and b's panels in L2.
  if (p.split_k == 1 && !p.stream_k())
    args.epilogue |= HEXIR_EPILOGUE_STREAM;

  const unsigned grid_x = p.tiles_m * p.tiles_n;
  hexir_status_t status;
  if (p.variant != kGuarded) {
    CUtensorMap map_a, map_b;
    const cuuint64_t a_dims[2] = {k, m};
    const cuuint64_t a_strides[1] = {static_cast<cuuint64_t>(lda) * 8};
    const cuuint32_t a_box[2] = {8, p.bm};
    const cuuint64_t b_dims[2] = {n, k};
    const cuuint64_t b_strides[1] = {static_cast<cuuint64_t>(n) * 8};
    const cuuint32_t b_box[2] = {16, HEXIR_LINEAR_BK};
    const cuuint32_t unit[2] = {1, 1};
    CUresult r = d.TensorMapEncodeTiled(
        &map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(a),
        a_dims, a_strides, a_box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
      r = d.TensorMapEncodeTiled(
          &map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(b),
          b_dims, b_strides, b_box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(error, cuda_message("cuTensorMapEncodeTiled", r));
    void *params[] = {&map_a, &map_b, &args};
    if (p.stream_k()) {
      status = launch(lib->linear_tma_sk, p.sk_grid, 1, HEXIR_LINEAR_THREADS,
                      HEXIR_LINEAR_SMEM_BYTES, stream, params,
                      "launch hexir_linear_f64_tma_sk", error);
      const unsigned sk_tiles = p.tiles_m * p.tiles_n - p.sk_dp_tiles;
      void *fix_params[] = {&args};
      if (status == HEXIR_OK)
        status = launch_after(lib->sk_fixup, sk_tiles, HEXIR_SK_FIXUP_PARTS, 256,
                              stream, fix_params,
                              "launch hexir_linear_f64_sk_fixup", error);
      d.EventRecord(dev->ws_ready, stream);
      return status;
    }
    CUfunction fn = lib->linear_tma;
    unsigned smem = HEXIR_LINEAR_SMEM_BYTES;
    const char *what = "launch hexir_linear_f64_tma";
    if (p.variant == kTma16) {
      fn = lib->linear_tma_m16;
      smem = HEXIR_LINEAR_M16_SMEM_BYTES;
      what = "launch hexir_linear_f64_tma_m16";
    } else if (p.variant == kTma64) {
      fn = lib->linear_tma_m64;
      smem = HEXIR_LINEAR_M64_SMEM_BYTES;
      what = "launch hexir_linear_f64_tma_m64";
    }
    status = launch(fn, grid_x, p.split_k, HEXIR_LINEAR_THREADS, smem, stream,
                    params, what, error);
  } else {
    void *params[] = {&args};
    status = launch(lib->linear_guarded, grid_x, p.split_k,
                    HEXIR_LINEAR_G_THREADS, HEXIR_LINEAR_G_SMEM_BYTES, stream,
                    params, "launch hexir_linear_f64_guarded", error);
  }
  if (status != HEXIR_OK || p.split_k == 1)
    return status;

  hexir_reduce_args_t red;
  red.partials = reinterpret_cast<const double *>(dev->workspace);
  red.c = c;
  red.count = static_cast<uint64_t>(m) * n;
  red.split = p.split_k;
  red.epilogue = args.epilogue;
  red.addend = addend;
  void *params[] = {&red};
  const uint64_t want = (red.count + 255) / 256;
  const unsigned grid = static_cast<unsigned>(std::max<uint64_t>(
      1, std::min<uint64_t>(want, static_cast<uint64_t>(dev->sm_count) * 8)));
  status = launch_after(lib->splitk_reduce, grid, 1, 256, stream, params,
                        "launch hexir_linear_f64_splitk_reduce", error);
  d.EventRecord(dev->ws_ready, stream);
  return status;
}

hexir_status_t launch_relu(DeviceState *dev, KernelLib *lib, const double *x,
                           double *y, size_t n, CUstream stream,
                           std::string *error) {
  if (n == 0)
    return HEXIR_OK;
  if (!x || !y)
    return fail(error, "relu: null pointer", HEXIR_ERROR_INVALID_ARGUMENT);
  hexir_elementwise_args_t args{x, nullptr, y, static_cast<uint64_t>(n)};
  void *params[] = {&args};
  return launch(lib->relu, stream_grid(dev, n / 2), 1, 256, 0, stream, params,
                "launch hexir_relu_f64", error);
}

hexir_status_t launch_add(DeviceState *dev, KernelLib *lib, const double *a,
                          const double *b, double *c, size_t n, CUstream stream,
                          std::string *error) {
  if (n == 0)
    return HEXIR_OK;
  if (!a || !b || !c)
    return fail(error, "add: null pointer", HEXIR_ERROR_INVALID_ARGUMENT);
  hexir_elementwise_args_t args{a, b, c, static_cast<uint64_t>(n)};
  void *params[] = {&args};
  return launch(lib->add, stream_grid(dev, n / 2), 1, 256, 0, stream, params,
                "launch hexir_add_f64", error);
}

hexir_status_t launch_activation(DeviceState *dev, KernelLib *lib, uint32_t op,
                                 const double *x, double *y, uint64_t rows,
                                 uint32_t cols, CUstream stream,
                                 std::string *error) {
  if (op < HEXIR_ACT_LEAKY_RELU || op > HEXIR_ACT_MISH)
    return fail(error, "activation: unknown op " + std::to_string(op),
                HEXIR_ERROR_INVALID_ARGUMENT);
  const uint64_t count = rows * cols;
  if (cols && count / cols != rows)
    return fail(error, "activation: rows x cols overflows",
                HEXIR_ERROR_INVALID_ARGUMENT);
  if (count == 0)
    return HEXIR_OK;
  if (!x || !y)
    return fail(error, "activation: null pointer", HEXIR_ERROR_INVALID_ARGUMENT);
  if (!lib->softmax_warp)
    return fail(error, "kernel library image lacks the activation kernels",
                HEXIR_ERROR_UNIMPLEMENTED);
  hexir_activation_args_t args{x, y, count, rows, cols, op, kWaitTimeoutNs};
  void *params[] = {&args};
  if (op != HEXIR_ACT_SOFTMAX)
    return launch(lib->activation[op - 7], stream_grid(dev, count / 2), 1, 256,
                  0, stream, params, "launch activation kernel", error);
  // Softmax: one row per warp or per block; blocks beyond the resident ones
  // queue, which balances rows of uneven cost.
  const uint64_t cap = 1u << 20;
  if (cols <= HEXIR_SOFTMAX_WARP_COLS) {
    const uint64_t blocks = std::min<uint64_t>((rows + 7) / 8, cap);
    return launch(lib->softmax_warp, static_cast<unsigned>(blocks), 1, 256, 0,
                  stream, params, "launch hexir_softmax_warp_f64", error);
  }
  // Even rows from a 16-byte aligned x start 16-byte aligned: the persistent
  // blocks that prefetch each next row with a bulk copy (two per SM for
  // rows up to 8192, one above).
  const bool bulk = cols % 2 == 0 && cols <= HEXIR_SOFTMAX_B512_COLS &&
                    (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                    lib->softmax_bulk256 && lib->softmax_bulk512;
  const uint64_t sms = static_cast<uint64_t>(std::max(dev->sm_count, 1));
  if (bulk && cols <= HEXIR_SOFTMAX_S2K_COLS && lib->softmax_bulk_s2k)
    return launch(lib->softmax_bulk_s2k,
                  static_cast<unsigned>(std::min<uint64_t>(rows, 5 * sms)), 1,
                  256, cols * 8u, stream, params,
                  "launch hexir_softmax_bulk_s2k_f64", error);
  if (bulk && cols <= HEXIR_SOFTMAX_S4K_COLS && lib->softmax_bulk_s4k)
    return launch(lib->softmax_bulk_s4k,
                  static_cast<unsigned>(std::min<uint64_t>(rows, 3 * sms)), 1,
                  256, cols * 8u, stream, params,
                  "launch hexir_softmax_bulk_s4k_f64", error);
  // Long even rows, 28674-65536 columns: a cluster of ceil(cols / 8192)
  // CTAs per row (4-8), each holding a segment at least 7/8 full, two CTAs
  // per SM.  Each row costs the cluster two barriers (~3.5 us with the
  // reductions), so shorter rows, whose segments would be part empty, stay
  // with the per-row blocks and the three-pass block.
  const bool clustered = cols % 2 == 0 && cols > 3u * HEXIR_SOFTMAX_B256_COLS +
                                                     HEXIR_SOFTMAX_B256_COLS / 2 &&
                         cols <= 8u * HEXIR_SOFTMAX_B256_COLS &&
                         (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                         lib->softmax_cluster[0] && driver().LaunchKernelEx;
  if (clustered) {
    const unsigned cl = (cols + HEXIR_SOFTMAX_B256_COLS - 1) / HEXIR_SOFTMAX_B256_COLS;
    const uint32_t seg = ((cols + cl - 1) / cl + 1u) & ~1u;
    CUfunction fn = lib->softmax_cluster[cl - 4];
    // Persistent clusters, all resident at once (a cluster that waited for
    // another to finish would add its whole share of rows to the time).
    unsigned resident = max_active_clusters(fn, cl, 256, seg * 8u);
    if (!resident)
      resident = static_cast<unsigned>(2 * sms / cl);
    const uint64_t clusters =
        std::max<uint64_t>(1, std::min<uint64_t>(rows, resident));
    return launch_cluster(fn,
                          static_cast<unsigned>(clusters * cl), cl, 256,
                          seg * 8u, stream, params,
                          "launch hexir_softmax_cluster_f64", error);
  }
  if (bulk && cols <= HEXIR_SOFTMAX_B256_COLS)
    return launch(lib->softmax_bulk256,
                  static_cast<unsigned>(std::min<uint64_t>(rows, 2 * sms)), 1,
                  256, cols * 8u, stream, params,
                  "launch hexir_softmax_bulk256_f64", error);
  if (bulk)
    return launch(lib->softmax_bulk512,
                  static_cast<unsigned>(std::min<uint64_t>(rows, sms)), 1, 512,
                  cols * 8u, stream, params, "launch hexir_softmax_bulk512_f64",
                  error);
  const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>(rows, cap));
  if (cols <= HEXIR_SOFTMAX_B256_COLS)
    return launch(lib->softmax_b256, blocks, 1, 256, 0, stream, params,
                  "launch hexir_softmax_b256_f64", error);
  if (cols <= HEXIR_SOFTMAX_B512_COLS)
    return launch(lib->softmax_b512, blocks, 1, 512, 0, stream, params,
                  "launch hexir_softmax_b512_f64", error);
  return launch(lib->softmax_wide, blocks, 1, 512, 0, stream, params,
                "launch hexir_softmax_wide_f64", error);
}

hexir_status_t check_device(DeviceState *dev, CUstream stream,
                            std::string *error) {
  const Driver &d = driver();
  ContextGuard guard(dev->context);
  CUresult r = d.StreamSynchronize(stream);
  if (r != CUDA_SUCCESS)
    return fail(error, cuda_message("kernel execution", r));
  std::lock_guard<std::mutex> lock(dev->mu);
  unsigned int bits = 0;
  for (auto &entry : dev->libs) {
    KernelLib *lib = entry.second.get();
    unsigned int word = 0;
    r = d.MemcpyDtoHAsync(&word, lib->error_word, sizeof(word), stream);
    if (r == CUDA_SUCCESS)
      r = d.StreamSynchronize(stream);
    if (r != CUDA_SUCCESS)
      return fail(error, cuda_message("reading the device error word", r));
    if (word) {
      bits |= word;
      d.MemsetD8Async(lib->error_word, 0, sizeof(word), stream);
      d.StreamSynchronize(stream);
    }
  }
  if (bits & HEXIR_KERR_WAIT_TIMEOUT)
    return fail(error, "a kernel pipeline wait ran out of time (device error "
                       "word " + std::to_string(bits) + ")");
  if (bits)
    return fail(error, "a kernel reported device error word " +
                           std::to_string(bits));
  return HEXIR_OK;
}

}  // namespace hexir

// ---- kernel-level C ABI --------------------------------------------------

using namespace hexir;

namespace {

struct Call {
  DeviceState *dev = nullptr;
  KernelLib *lib = nullptr;
  std::string error;
  bool open(int ordinal) {
    dev = device_state(ordinal, &error);
    if (!dev)
      return false;
    lib = embedded_library(dev, &error);
    return lib != nullptr;
  }
  hexir_status_t finish(hexir_status_t status) {
    if (status != HEXIR_OK)
      set_last_error(error.empty() ? hexir_status_string(status) : error);
    return status;
  }
};

}  // namespace

extern "C" hexir_status_t hexir_cuda_matmul_f64(int ordinal, const double *a,
                                                const double *b, double *c,
                                                uint32_t m, uint32_t n,
                                                uint32_t k, uint32_t flags,
                                                void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  ContextGuard guard(call.dev->context);
  return call.finish(launch_matmul(call.dev, call.lib, a, b, c, m, n, k, flags,
                                   static_cast<CUstream>(stream), &call.error));
}

extern "C" hexir_status_t hexir_cuda_matmul_acc_f64(
    int ordinal, const double *a, uint32_t lda, const double *b,
    const double *c_in, double *c, uint32_t m, uint32_t n, uint32_t k,
    uint32_t flags, void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  // Never split over k, with or without c_in: every piece of a product
  // computed in k ranges must sum its range in one pass.
  if (((flags >> 16) & 0xFFu) > 1) {
    call.error = "matmul: a continued sum cannot be split over k";
    return call.finish(HEXIR_ERROR_INVALID_ARGUMENT);
  }
  flags = (flags & ~0xFF0000u) | HEXIR_MATMUL_SPLIT_K(1);
  ContextGuard guard(call.dev->context);
  return call.finish(launch_matmul(call.dev, call.lib, a, b, c, m, n, k, flags,
                                   static_cast<CUstream>(stream), &call.error,
                                   lda, c_in));
}

extern "C" hexir_status_t hexir_cuda_matmul_add_f64(
    int ordinal, const double *a, const double *b, const double *addend,
    double *c, uint32_t m, uint32_t n, uint32_t k, uint32_t flags,
    void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  if (!addend && m && n) {
    call.error = "matmul_add: null addend";
    return call.finish(HEXIR_ERROR_INVALID_ARGUMENT);
  }
  ContextGuard guard(call.dev->context);
  return call.finish(launch_matmul(call.dev, call.lib, a, b, c, m, n, k, flags,
                                   static_cast<CUstream>(stream), &call.error,
                                   0, nullptr, addend));
}

extern "C" hexir_status_t hexir_cuda_add_f64(int ordinal, const double *a,
                                             const double *b, double *c,
                                             size_t n, void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  ContextGuard guard(call.dev->context);
  return call.finish(launch_add(call.dev, call.lib, a, b, c, n,
                                static_cast<CUstream>(stream), &call.error));
}

extern "C" hexir_status_t hexir_cuda_relu_f64(int ordinal, const double *x,
                                              double *y, size_t n,
                                              void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  ContextGuard guard(call.dev->context);
  return call.finish(launch_relu(call.dev, call.lib, x, y, n,
                                 static_cast<CUstream>(stream), &call.error));
}

extern "C" hexir_status_t hexir_cuda_activation_f64(int ordinal, uint32_t op,
                                                    const double *x, double *y,
                                                    uint64_t rows, uint32_t cols,
                                                    void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  ContextGuard guard(call.dev->context);
  return call.finish(launch_activation(call.dev, call.lib, op, x, y, rows, cols,
                                       static_cast<CUstream>(stream),
                                       &call.error));
}

extern "C" hexir_status_t hexir_cuda_synchronize(int ordinal, void *stream) {
  Call call;
  call.dev = device_state(ordinal, &call.error);
  if (!call.dev)
    return call.finish(HEXIR_ERROR_DEVICE);
  return call.finish(
      check_device(call.dev, static_cast<CUstream>(stream), &call.error));
}

extern "C" hexir_status_t hexir_cuda_matmul_plan(int ordinal, const double *a,
                                                 const double *b, double *c,
                                                 uint32_t m, uint32_t n,
                                                 uint32_t k, uint32_t flags,
                                                 int *variant,
                                                 uint32_t *split_k) {
  std::string error;
  DeviceState *dev = device_state(ordinal, &error);
  MatmulPlan p = plan_matmul(dev, a, b, c, m, n, k, flags);
  if (variant)
    *variant = p.variant;
  if (split_k)
    *split_k = p.stream_k() ? p.sk_grid : p.split_k;
  return HEXIR_OK;
}

extern "C" hexir_status_t hexir_cuda_baseline_reference_schedule_f64(
    int ordinal, const double *a, const double *b, double *c, uint32_t m,
    uint32_t n, uint32_t k, void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  if (!call.lib->baseline_schedule) {
    call.error = "kernel image lacks hexir_baseline_reference_schedule_f64";
    return call.finish(HEXIR_ERROR_NOT_FOUND);
  }
  // The generated kernel's grid puts the rows on grid.y, which stops at
  // 65535: larger m cannot launch in the reference either.
  if (m > 65535u) {
    call.error = "reference schedule: m > 65535 rows does not fit grid.y";
    return call.finish(HEXIR_ERROR_INVALID_ARGUMENT);
  }
  if (!m || !n)
    return HEXIR_OK;
  if (!a || !b || !c) {
    call.error = "reference schedule: null operand";
    return call.finish(HEXIR_ERROR_INVALID_ARGUMENT);
  }
  uint32_t bs = 256;
  while (bs > 1 && n % bs)
    bs /= 2;
  ContextGuard guard(call.dev->context);
  void *params[] = {&a, &b, &c, &n, &k};
  return call.finish(launch(call.lib->baseline_schedule, n / bs, m, bs, 0,
                            static_cast<CUstream>(stream), params,
                            "launch hexir_baseline_reference_schedule_f64",
                            &call.error));
}

extern "C" hexir_status_t hexir_cuda_dmma_probe(int ordinal, double *out,
                                                uint32_t blocks, uint32_t iters,
                                                void *stream, double *flops) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  if (!out || blocks == 0)
    return call.finish(HEXIR_ERROR_INVALID_ARGUMENT);
  ContextGuard guard(call.dev->context);
  void *params[] = {&out, &iters};
  hexir_status_t s = launch(call.lib->dmma_probe, blocks, 1, 256, 0,
                            static_cast<CUstream>(stream), params,
                            "launch hexir_dmma_peak_probe", &call.error);
  if (flops)
    *flops = static_cast<double>(blocks) * (256 / 32) * iters * 8.0 *
             (2.0 * 16 * 8 * 8);
  return call.finish(s);
}

extern "C" hexir_status_t hexir_cuda_wait_probe(int ordinal,
                                               uint64_t timeout_ns,
                                               void *stream) {
  Call call;
  if (!call.open(ordinal))
    return call.finish(HEXIR_ERROR_DEVICE);
  ContextGuard guard(call.dev->context);
  void *params[] = {&timeout_ns};
  return call.finish(launch(call.lib->wait_probe, 1, 1, 32, 0,
                            static_cast<CUstream>(stream), params,
                            "launch hexir_wait_timeout_probe", &call.error));
}

extern "C" uint64_t hexir_cuda_launch_count(void) {
  return g_launches.load(std::memory_order_relaxed);
}

extern "C" int hexir_cuda_sm_count(int ordinal) {
  std::string error;
  DeviceState *dev = device_state(ordinal, &error);
  return dev ? dev->sm_count : 0;
}

extern "C" hexir_status_t hexir_cuda_kernel_image(const void **data,
                                                  size_t *size) {
  if (!data || !size)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *data = embedded_image_data();
  *size = embedded_image_size();
  return HEXIR_OK;
}

extern "C" const char *hexir_cuda_last_error(void) {
  return g_last_error.c_str();
}
