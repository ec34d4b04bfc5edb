// elementwise_f64.cu -- the reference relu and add over a flat f64 range,
// bit-for-bit equal to runtime/src/kernels/reference_kernels.c:15-23:
//   relu: y[i] = x[i] > 0.0 ? x[i] : 0.0   (NaN -> +0.0, -0.0 -> +0.0)
//   add:  c[i] = a[i] + b[i]               (one IEEE round-to-nearest add)
//
// Pure HBM streams: 16-byte vector loads and stores with the streaming cache
// hint, four independent vectors in flight per thread, grid-stride over a
// grid sized by the host to a multiple of the SM count.  A scalar path covers
// pointers that are not 16-byte aligned and the odd last element.

#include "common.cuh"

using namespace hexir;

namespace {

struct ReluOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    return relu_ref(x);
  }
};
struct AddOp {
  __device__ __forceinline__ double operator()(double x, double y) const {
    return __dadd_rn(x, y);
  }
};

template <bool BINARY, typename Op>
__device__ __forceinline__ void stream_f64(const hexir_elementwise_args_t &p,
                                           Op op) {
  const uint64_t n = p.count;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(p.x) |
                     reinterpret_cast<uintptr_t>(p.out) |
                     (BINARY ? reinterpret_cast<uintptr_t>(p.y) : 0)) &
                    15u) == 0;
  if (!vec) {
    for (uint64_t i = tid; i < n; i += stride)
      p.out[i] = op(p.x[i], BINARY ? p.y[i] : 0.0);
    return;
  }
  const uint64_t pairs = n >> 1;
  const double2 *__restrict__ x2 = reinterpret_cast<const double2 *>(p.x);
  const double2 *__restrict__ y2 = reinterpret_cast<const double2 *>(p.y);
  double2 *__restrict__ o2 = reinterpret_cast<double2 *>(p.out);
  uint64_t i = tid;
  for (; i + 3 * stride < pairs; i += 4 * stride) {
    double2 v[4], w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = __ldcs(x2 + i + u * stride);
      if (BINARY)
        w[u] = __ldcs(y2 + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      double2 r;
      r.x = op(v[u].x, BINARY ? w[u].x : 0.0);
      r.y = op(v[u].y, BINARY ? w[u].y : 0.0);
      __stcs(o2 + i + u * stride, r);
    }
  }
  for (; i < pairs; i += stride) {
    const double2 v = __ldcs(x2 + i);
    double2 w = make_double2(0.0, 0.0);
    if (BINARY)
      w = __ldcs(y2 + i);
    double2 r;
    r.x = op(v.x, w.x);
    r.y = op(v.y, w.y);
    __stcs(o2 + i, r);
  }
  if ((n & 1) && tid == 0)
    p.out[n - 1] = op(p.x[n - 1], BINARY ? p.y[n - 1] : 0.0);
}

}  // namespace

extern "C" __global__ void __launch_bounds__(256)
    hexir_relu_f64(const hexir_elementwise_args_t args) {
  stream_f64<false>(args, ReluOp{});
}

extern "C" __global__ void __launch_bounds__(256)
    hexir_add_f64(const hexir_elementwise_args_t args) {
  stream_f64<true>(args, AddOp{});
}
