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
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

#include "hal_internal.h"

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

void cpu_add_f64(const double *a, const double *b, double *c, size_t n) {
  for (size_t i = 0; i < n; ++i)
    c[i] = a[i] + b[i];
}

void cpu_relu_f64(const double *x, double *y, size_t n) {
  for (size_t i = 0; i < n; ++i)
    y[i] = x[i] > 0.0 ? x[i] : 0.0;
}

}  // namespace hexir
