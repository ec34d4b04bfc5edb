// cpu_kernels.cc -- bodies of cpu-placed dispatches.
//
// The CPU backend is part of the surface being replaced: a module whose ops
// are placed on cpu runs them on the host, exactly as the reference runtime
// does with runtime/src/kernels/reference_kernels.c:3-23.  Same arithmetic:
// each output element is a sequential k loop starting from 0.0 with a
// separate multiply and add (this file is compiled with -ffp-contract=off),
// so results are bit-identical to the reference CPU path.  Rows are spread
// over host threads; that changes no element's summation order.
//
// cuda-placed dispatches never come here: the VM refuses them on a CPU device.

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "hal_internal.h"
#include "hexir_runtime/program.h"

namespace hexir {

namespace {

template <typename Fn>
void parallel_rows(uint64_t rows, uint64_t work_per_row, Fn fn) {
  unsigned threads = std::max(1u, std::thread::hardware_concurrency());
  // Small problems stay on the calling thread.
  if (rows < 2 || rows * work_per_row < (1u << 22))
    threads = 1;
  threads = static_cast<unsigned>(std::min<uint64_t>(threads, rows));
  if (threads <= 1) {
    fn(0, rows);
    return;
  }
  std::vector<std::thread> pool;
  const uint64_t per = (rows + threads - 1) / threads;
  for (unsigned t = 0; t < threads; ++t) {
    const uint64_t begin = t * per, end = std::min(rows, begin + per);
    if (begin >= end)
      break;
    pool.emplace_back([=] { fn(begin, end); });
  }
  for (auto &th : pool)
    th.join();
}

}  // namespace

void cpu_matmul_f64(const double *a, const double *b, double *c, uint32_t m,
                    uint32_t n, uint32_t k) {
  parallel_rows(m, static_cast<uint64_t>(n) * k, [=](uint64_t r0, uint64_t r1) {
    for (uint64_t i = r0; i < r1; ++i) {
      for (uint32_t j = 0; j < n; ++j) {
        double acc = 0.0;
        for (uint32_t p = 0; p < k; ++p)
          acc += a[i * k + p] * b[static_cast<size_t>(p) * n + j];
        c[i * n + j] = acc;
      }
    }
  });
}

// The elementwise ops in ranges of kElementsPerRange over the host threads:
// they are memory-bound, so one thread leaves most of the host's bandwidth
// unused on a tensor of hundreds of MiB.  Each element's operation is the
// same, so the bits are too.
constexpr uint64_t kElementsPerRange = 1u << 16;

void cpu_add_f64(const double *a, const double *b, double *c, size_t n) {
  const uint64_t ranges = (n + kElementsPerRange - 1) / kElementsPerRange;
  parallel_rows(ranges, kElementsPerRange, [=](uint64_t r0, uint64_t r1) {
    const size_t end = std::min<size_t>(n, r1 * kElementsPerRange);
    for (size_t i = r0 * kElementsPerRange; i < end; ++i)
      c[i] = a[i] + b[i];
  });
}

void parallel_copy(void *dst, const void *src, size_t bytes) {
  constexpr uint64_t kBytesPerRange = 1u << 20;
  const uint64_t ranges = (bytes + kBytesPerRange - 1) / kBytesPerRange;
  // Threads for copies of 4 MiB and more (parallel_rows' 2^22 threshold,
  // counted in bytes).
  parallel_rows(ranges, kBytesPerRange, [=](uint64_t r0, uint64_t r1) {
    const size_t b0 = r0 * kBytesPerRange;
    const size_t b1 = std::min<size_t>(bytes, r1 * kBytesPerRange);
    std::memcpy(static_cast<char *>(dst) + b0,
                static_cast<const char *>(src) + b0, b1 - b0);
  });
}

void cpu_relu_f64(const double *x, double *y, size_t n) {
  const uint64_t ranges = (n + kElementsPerRange - 1) / kElementsPerRange;
  parallel_rows(ranges, kElementsPerRange, [=](uint64_t r0, uint64_t r1) {
    const size_t end = std::min<size_t>(n, r1 * kElementsPerRange);
    for (size_t i = r0 * kElementsPerRange; i < end; ++i)
      y[i] = x[i] > 0.0 ? x[i] : 0.0;
  });
}

// The activations the reference dialect declares without lowering
// (include/hexir/Dialect/Hexir/IR/HexirOps.td:189-308), as the GPU kernels
// evaluate them: each op description written in a form that keeps its
// relative accuracy (gelu through erfc, softplus split at 0), leaky_relu's
// alpha 0.01 and elu's alpha 1.0 fixed because the ops carry no attribute.
// Softmax subtracts the row maximum (NaN skipped by the compare) and sums the
// row left to right.
namespace {

double softplus(double x) {
  return x > 0.0 ? x + std::log1p(std::exp(-x)) : std::log1p(std::exp(x));
}

double activation(uint32_t kind, double x) {
  switch (kind) {
  case HEXIR_KERNEL_LEAKY_RELU: return x > 0.0 ? x : 0.01 * x;
  case HEXIR_KERNEL_ELU: return x > 0.0 ? x : 1.0 * std::expm1(x);
  case HEXIR_KERNEL_SIGMOID: return 1.0 / (1.0 + std::exp(-x));
  case HEXIR_KERNEL_TANH: return std::tanh(x);
  case HEXIR_KERNEL_GELU:
    return (0.5 * x) * std::erfc(-x * 0.70710678118654752440);
  case HEXIR_KERNEL_SWISH: return x / (1.0 + std::exp(-x));
  case HEXIR_KERNEL_MISH: return x * std::tanh(softplus(x));
  }
  return x;
}

}  // namespace

void cpu_activation_f64(uint32_t kind, const double *x, double *y,
                        uint64_t rows, uint64_t cols) {
  if (kind == HEXIR_KERNEL_SOFTMAX) {
    parallel_rows(rows, cols * 8, [=](uint64_t r0, uint64_t r1) {
      for (uint64_t r = r0; r < r1; ++r) {
        const double *xr = x + r * cols;
        double *yr = y + r * cols;
        double m = -HUGE_VAL;
        for (uint64_t j = 0; j < cols; ++j)
          m = xr[j] > m ? xr[j] : m;
        double s = 0.0;
        for (uint64_t j = 0; j < cols; ++j) {
          yr[j] = std::exp(xr[j] - m);
          s += yr[j];
        }
        for (uint64_t j = 0; j < cols; ++j)
          yr[j] = yr[j] / s;
      }
    });
    return;
  }
  const uint64_t n = rows * cols;
  const uint64_t chunk = 1u << 16;
  parallel_rows((n + chunk - 1) / chunk, chunk * 8, [=](uint64_t c0, uint64_t c1) {
    const uint64_t end = std::min(n, c1 * chunk);
    for (uint64_t i = c0 * chunk; i < end; ++i)
      y[i] = activation(kind, x[i]);
  });
}

}  // namespace hexir
