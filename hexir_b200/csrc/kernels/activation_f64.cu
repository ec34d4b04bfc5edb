// activation_f64.cu -- the hexir dialect's declared activations
// (include/hexir/Dialect/Hexir/IR/HexirOps.td:189-308) over f64 tensors:
//
//   leaky_relu  x > 0 ? x : 0.01 x          ("max(x, alpha * x)", alpha fixed)
//   elu         x > 0 ? x : 1.0 expm1(x)    ("alpha * (exp(x) - 1)", alpha fixed)
//   sigmoid     1 / (1 + exp(-x))
//   tanh        tanh(x), as -u / (2 + u), u = expm1(-2|x|) (see TanhOp)
//   softmax     exp(x - max) / sum exp(x - max) along each row
//   gelu        0.5 x erfc(-x / sqrt 2)     (= x 0.5 (1 + erf(x / sqrt 2)),
//                                            without the cancellation of 1 + erf
//                                            for negative x; see GeluOp)
//   swish       x / (1 + exp(-x))           (= x sigmoid(x), one rounding)
//   mish        x tanh(softplus(x)), evaluated with one exp and one divide:
//               tanh(log(1 + e^x)) = ((1 + e^x)^2 - 1) / ((1 + e^x)^2 + 1), so
//               with u = e^x for x <= 0:   q = u (u + 2) / (u (u + 2) + 2)
//               and  u = e^-x for x > 0:   q = (1 + 2u) / (1 + 2u + 2u^2)
//               (every term positive, nothing overflows), mish = x q.  Within
//               4 ulp of the exact value, as the exp / log1p / tanh chain is
//               within 3; the chain costs about six times as much here.
//
// The reference declares these ops but lowers none of them; the formulas
// above are its op descriptions written in forms that keep their relative
// accuracy over the whole f64 range.  The host backend (cpu_kernels.cc)
// evaluates them with the C library's functions (mish as the literal
// x tanh(softplus(x)), softmax dividing by the sum), so the two agree to a
// few units in the last place.  Every add, multiply and
// divide here is an explicit round-to-nearest intrinsic so that no fused
// multiply-add is formed across the inlined math functions.
//
// Elementwise ops run on the relu/add stream loop (16-byte streaming loads and
// stores, four vectors in flight per thread).  Softmax keeps each row in
// registers (one read and one write of the row): a warp per row up to 1024
// columns; above that, for even rows starting 16-byte aligned, persistent
// blocks that bulk-copy their next row into shared memory while the current
// one computes (up to 8192 / 16384 columns with 256 / 512 threads); for other
// rows one 256- or 512-thread block per row; and a three-pass block per row
// beyond 16384 columns.  It scales by one correctly rounded reciprocal of the
// row sum instead of dividing every element.
//
// FP64 arithmetic, not HBM, bounds the transcendental ones on B200 (gelu's
// erfc, tanh, softmax's exp): each element costs tens of FP64 instructions.

namespace {

__device__ __forceinline__ double neg_inf() {
  return __longlong_as_double(static_cast<long long>(0xfff0000000000000ull));
}

// e^z for z <= 0, built from its parts (no call, no branch):
//  - z = k ln2 + r, |r| <= ln2 / 2: k by adding and subtracting 1.5 * 2^52
//    (round to nearest), r by Cody and Waite's two-part ln 2 (the first fma
//    is exact);
//  - expm1(r) by its Taylor series to r^13 / 13! (truncation below 2^-56
//    relative for |r| <= ln2 / 2), Horner in fma.
// neg_exp_parts returns p = expm1(r) and k, for z in [-746, 0] or NaN.
// Measured on B200 against CUDA's functions in the same kernels: in place of
// expm1 it wins (tanh, elu), and so it does beside the divide-free quotient
// in mish; sigmoid, swish and softmax stay faster with CUDA's exp (and
// sigmoid and swish with the IEEE divide: with the quotient below CUDA's exp
// spilled registers there).  The order of the differences was 5-15 %.
__device__ __forceinline__ double neg_exp_parts(double z, int &k) {
  const double shifter = 0x1.8p52;
  const double t = __fma_rn(z, 0x1.71547652b82fep+0, shifter);  // z / ln2
  const double kd = __dsub_rn(t, shifter);
  k = __double2loint(t);
  double r = __fma_rn(-kd, 0x1.62e42fefa39efp-1, z);
  r = __fma_rn(-kd, 0x1.abc9e3b39803fp-56, r);
  double q = 0x1.6124613a86d09p-33;  // 1 / 13!
  q = __fma_rn(q, r, 0x1.1eed8eff8d898p-29);
  q = __fma_rn(q, r, 0x1.ae64567f544e4p-26);
  q = __fma_rn(q, r, 0x1.27e4fb7789f5cp-22);
  q = __fma_rn(q, r, 0x1.71de3a556c734p-19);
  q = __fma_rn(q, r, 0x1.a01a01a01a01ap-16);
  q = __fma_rn(q, r, 0x1.a01a01a01a01ap-13);
  q = __fma_rn(q, r, 0x1.6c16c16c16c17p-10);
  q = __fma_rn(q, r, 0x1.1111111111111p-7);
  q = __fma_rn(q, r, 0x1.5555555555555p-5);
  q = __fma_rn(q, r, 0x1.5555555555555p-3);
  q = __fma_rn(q, r, 0.5);                                      // 1 / 2!
  return __fma_rn(__dmul_rn(r, r), q, r);
}

// 2^k for k in [-1022, 1023], in the exponent bits.
__device__ __forceinline__ double pow2i(int k) {
  return __hiloint2double((k + 1023) << 20, 0);
}

// e^z for z <= 0 (below -746 it is 0; NaN passes): 2^k (1 + p), scaled in
// two halves of k so that results in the subnormal range round once.
__device__ __forceinline__ double exp_neg(double z) {
  int k;
  const double p = neg_exp_parts(z < -746.0 ? -746.0 : z, k);
  const int k1 = k >> 1;
  return __dmul_rn(__dmul_rn(__dadd_rn(1.0, p), pow2i(k1)), pow2i(k - k1));
}

// expm1(z) for z in [-40, 0] or NaN: 2^k p + (2^k - 1) in one fma.
__device__ __forceinline__ double expm1_neg_core(double z) {
  int k;
  const double p = neg_exp_parts(z, k);
  const double s = pow2i(k);
  return __fma_rn(s, p, __dsub_rn(s, 1.0));
}

// expm1(z) for any z <= 0 (below -40 it rounds to -1; NaN passes).
__device__ __forceinline__ double expm1_neg(double z) {
  return expm1_neg_core(z < -40.0 ? -40.0 : z);
}

__device__ __forceinline__ double rcp_estimate(double d) {
  double r;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(d));
  return r;
}

// n / d for a normal d > 0 and a finite n, without the IEEE divide: one
// Newton-Raphson step on the hardware reciprocal estimate, then one
// Markstein correction of the quotient.  The error after both is about the
// estimate's to the fourth power, so any estimate of 20 bits or more gives
// the quotient of the exact reciprocal (on B200 the results equal those of
// two Newton steps on 2^28 inputs): within an ulp, not always the correctly
// rounded one.  A zero quotient comes out +0.
__device__ __forceinline__ double quotient(double n, double d) {
  double rc = rcp_estimate(d);
  rc = __fma_rn(rc, __fma_rn(-d, rc, 1.0), rc);
  const double q0 = __dmul_rn(n, rc);
  return __fma_rn(rc, __fma_rn(-d, q0, n), q0);
}

struct LeakyReluOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    return x > 0.0 ? x : __dmul_rn(HEXIR_LEAKY_RELU_ALPHA, x);
  }
};
// elu(x) = x for x > 0, alpha expm1(x) below (alpha 1); +-0 and NaN pass
// through (expm1(+-0) = +-0).
struct EluOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    static_assert(HEXIR_ELU_ALPHA == 1.0, "expm1 below zero is scaled by 1");
    return x < 0.0 ? expm1_neg(x) : x;
  }
};
struct SigmoidOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
  }
};
// tanh(x) = sign(x) * -u / (2 + u) with u = expm1(-2|x|) in [-1, 0]
// (tanh|x| = (1 - e^{-2|x|}) / (1 + e^{-2|x|})), |x| capped at 20 (beyond
// 19.1 tanh rounds to 1; NaN passes), by expm1_neg and quotient above: no
// call and no branch, so every lane runs the same ~30 FP64 instructions.
// Within 3 ulp of the C library's tanh and 2.6 ulp of a 64-bit reference
// on 2 * 10^7 sampled inputs (normal, uniform to +-25, tiny, subnormal, the
// k boundaries); +-0 keeps its sign.  Measured 0.87 of copy bandwidth on
// B200, against 0.72 for expm1 and an IEEE divide: the kernel is bound by
// FP64 instruction issue, so each instruction saved shows.
struct TanhOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    const double ax = fabs(x);
    const double y = ax > 20.0 ? 20.0 : ax;
    const double u = expm1_neg_core(__dmul_rn(-2.0, y));  // -2y >= -40
    return copysign(quotient(-u, __dadd_rn(2.0, u)), x);  // d in [1, 2]
  }
};
// gelu(x) = (x / 2) erfc(-x / sqrt 2), the argument rounded as written:
// u = RN(|x| RN(1 / sqrt 2)); erfc(u) / 2 = R(u) e^{-u^2}, and gelu is
// x erfc(u) / 2 for x < 0 and x (1 - erfc(u) / 2) above (erfc(-u) =
// 2 - erfc(u)), so neither side cancels.  R(u) = erfc(u) e^{u^2} / 2 is a
// degree-9 polynomial on each of 228 intervals of width 1/8 over [0, 28.5)
// (gelu_table.inc, written by gelu_table_gen.c from the C library's erfcl
// in long double; relative error below 2.2e-16 as rounded); u^2 is carried
// as a double-double into exp_neg (CUDA's exp, a call on its wide path,
// made this kernel spill).  Every lane runs the same
// instructions: the interval picks the coefficients, from shared memory,
// not the code.  Within 3.9 ulp of the formula evaluated exactly and 5 ulp
// of the C library's erfc form, on 5 * 10^6 sampled inputs; CUDA's erfc
// cost about six times the instructions.
constexpr int kGeluIntervals = 228;
constexpr int kGeluRow = 10;
__device__ const double kGeluTable[kGeluIntervals][kGeluRow] = {
#include "gelu_table.inc"
};
struct GeluOp {
  const double *table;  // kGeluTable, staged in shared memory
  __device__ __forceinline__ double operator()(double x, double) const {
    const double u0 = __dmul_rn(fabs(x), 0.70710678118654752440);
    const double u = u0 > 28.5 ? 28.5 : u0;  // erfc(28.5) underflows; NaN passes
    int j = __double2int_rz(__dmul_rn(u, 8.0));
    j = min(max(j, 0), kGeluIntervals - 1);
    const double t = __fma_rn(u, 16.0, -static_cast<double>(2 * j + 1));
    const double2 *row = reinterpret_cast<const double2 *>(table + j * kGeluRow);
    const double2 c01 = row[0], c23 = row[1], c45 = row[2], c67 = row[3],
                  c89 = row[4];
    double p = __fma_rn(c89.y, t, c89.x);
    p = __fma_rn(p, t, c67.y);
    p = __fma_rn(p, t, c67.x);
    p = __fma_rn(p, t, c45.y);
    p = __fma_rn(p, t, c45.x);
    p = __fma_rn(p, t, c23.y);
    p = __fma_rn(p, t, c23.x);
    p = __fma_rn(p, t, c01.y);
    p = __fma_rn(p, t, c01.x);
    const double uu = __dmul_rn(u, u);
    const double lo = __fma_rn(u, u, -uu);  // u^2 = uu + lo exactly
    double e = exp_neg(-uu);
    e = __fma_rn(-lo, e, e);                  // e^{-uu} (1 - lo)
    const double q = __dmul_rn(p, e);         // erfc(u) / 2
    return __dmul_rn(x, x < 0.0 ? q : __dsub_rn(1.0, q));
  }
};
struct SwishOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    return __ddiv_rn(x, __dadd_rn(1.0, exp(-x)));
  }
};
struct MishOp {
  __device__ __forceinline__ double operator()(double x, double) const {
    const bool neg = x <= 0.0;
    const double u = exp_neg(-fabs(x));
    const double num = neg ? __dmul_rn(u, __dadd_rn(u, 2.0))
                           : __dadd_rn(1.0, __dmul_rn(2.0, u));
    const double den =
        __dadd_rn(num, neg ? 2.0 : __dmul_rn(__dmul_rn(2.0, u), u));
    return __dmul_rn(x, quotient(num, den));  // den in [1, 5]
  }
};

template <typename Op>
__device__ __forceinline__ void activation_stream(
    const hexir_activation_args_t &a, Op op) {
  const hexir_elementwise_args_t e{a.x, nullptr, a.out, a.count};
  stream_f64<false>(e, op);
}

// ---------------------------------------------------------------- softmax

struct MaxOp {
  __device__ __forceinline__ double operator()(double a, double b) const {
    return b > a ? b : a;
  }
};
struct SumOp {
  __device__ __forceinline__ double operator()(double a, double b) const {
    return __dadd_rn(a, b);
  }
};

// Butterfly over the warp: IEEE add and the compare-select max are
// commutative, so every lane ends with the same value.
template <typename Op>
__device__ __forceinline__ double warp_reduce(double v, Op op) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The block's reduction, the same value in every thread: warps reduce, then
// every thread folds the per-warp values in warp order.
template <int THREADS, typename Op>
__device__ __forceinline__ double block_reduce(double v, double *red, Op op) {
  v = warp_reduce(v, op);
  if ((threadIdx.x & 31) == 0)
    red[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = red[0];
#pragma unroll
  for (int w = 1; w < THREADS / 32; ++w)
    r = op(r, red[w]);
  __syncthreads();
  return r;
}

// One row per block, PER elements per thread kept in registers: one read and
// one write of the row.  The maximum skips NaN (x > m is false); a NaN or an
// infinity in the row makes the whole row NaN through exp(x - m), as in the
// host formula.
template <int THREADS, int PER>
__device__ __forceinline__ void softmax_rows_block(
    const hexir_activation_args_t &p) {
  __shared__ double red[THREADS / 32];
  const uint32_t cols = p.cols;
  for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const double *xr = p.x + row * cols;
    double *yr = p.out + row * cols;
    double v[PER];
    double m = neg_inf();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      v[i] = j < cols ? __ldcs(xr + j) : neg_inf();
      m = v[i] > m ? v[i] : m;
    }
    m = block_reduce<THREADS>(m, red, MaxOp{});
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      if (j < cols) {
        v[i] = exp(__dsub_rn(v[i], m));
        s = __dadd_rn(s, v[i]);
      }
    }
    const double rs = __drcp_rn(block_reduce<THREADS>(s, red, SumOp{}));
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      if (j < cols)
        __stcs(yr + j, __dmul_rn(v[i], rs));
    }
  }
}

// One row per warp, PER elements per lane.
template <int PER>
__device__ __forceinline__ void softmax_rows_warp(
    const hexir_activation_args_t &p) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
  const uint32_t cols = p.cols;
  for (uint64_t row = (static_cast<uint64_t>(blockIdx.x) * blockDim.x +
                       threadIdx.x) >> 5;
       row < p.rows; row += warps) {
    const double *xr = p.x + row * cols;
    double *yr = p.out + row * cols;
    double v[PER];
    double m = neg_inf();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = lane + i * 32;
      v[i] = j < cols ? __ldcs(xr + j) : neg_inf();
      m = v[i] > m ? v[i] : m;
    }
    m = warp_reduce(m, MaxOp{});
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = lane + i * 32;
      if (j < cols) {
        v[i] = exp(__dsub_rn(v[i], m));
        s = __dadd_rn(s, v[i]);
      }
    }
    const double rs = __drcp_rn(warp_reduce(s, SumOp{}));
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = lane + i * 32;
      if (j < cols)
        __stcs(yr + j, __dmul_rn(v[i], rs));
    }
  }
}

// Persistent blocks (rows blockIdx.x, + gridDim.x, ...), PER elements per
// thread in registers, and one row-sized shared buffer that the bulk-copy
// engine fills with the block's next row while the current one computes:
//   wait for row r in smem -> registers, maximum (block reduction; after it
//   no thread reads the buffer) -> one thread starts the copy of the next
//   row -> exp, sum, reciprocal, scaled stores of row r.
// The host runs it only for an even row length and a 16-byte aligned x, so
// every row starts 16-byte aligned and is a multiple of 16 bytes long.  A
// wait that runs out (timeout_ns) sets the error word and the whole block
// returns; the only copy in flight is the one that did not arrive.
template <int THREADS, int PER>
__device__ __forceinline__ void softmax_rows_bulk(
    const hexir_activation_args_t &p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ double red[THREADS / 32];
  __shared__ __align__(8) uint64_t bar;
  double *buf = reinterpret_cast<double *>(smem_raw);
  const uint32_t cols = p.cols;
  const uint32_t bytes = cols * 8u;
  uint64_t row = blockIdx.x;
  if (row >= p.rows)
    return;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_load(buf, p.x + row * cols, bytes, &bar);
  }
  uint32_t phase = 0;
  for (; row < p.rows; row += gridDim.x) {
    const bool arrived = mbar_wait_bounded(&bar, phase, p.timeout_ns);
    if (!__syncthreads_and(arrived))
      return;
    phase ^= 1u;
    double *yr = p.out + row * cols;
    double v[PER];
    double m = neg_inf();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      v[i] = j < cols ? buf[j] : neg_inf();
      m = v[i] > m ? v[i] : m;
    }
    m = block_reduce<THREADS>(m, red, MaxOp{});
    const uint64_t next = row + gridDim.x;
    if (threadIdx.x == 0 && next < p.rows) {
      mbar_arrive_expect_tx(&bar, bytes);
      bulk_load(buf, p.x + next * cols, bytes, &bar);
    }
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      if (j < cols) {
        v[i] = exp(__dsub_rn(v[i], m));
        s = __dadd_rn(s, v[i]);
      }
    }
    const double rs = __drcp_rn(block_reduce<THREADS>(s, red, SumOp{}));
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      if (j < cols)
        __stcs(yr + j, __dmul_rn(v[i], rs));
    }
  }
}

// Rows longer than one block holds, split over a thread-block cluster of CL
// CTAs: CTA r of the cluster holds columns [r seg, (r + 1) seg) of each row
// (seg = cols / CL rounded up to even), in registers and, for the next row,
// in its shared memory by bulk copy as in softmax_rows_bulk.  The row's
// maximum and sum are each reduced in the CTA, published in one shared f64
// of the CTA, and combined over the cluster in rank order through
// distributed shared memory between two cluster barriers per row.  One slot
// each is enough: a CTA writes its next maximum only after the second
// barrier of the row, which every peer reaches only after reading the first
// maximum, and its next sum only after the next row's first barrier, which
// every peer reaches only after reading this sum.  Every CTA of a cluster
// walks the same rows and executes the same barriers (a copy that times out
// marks the error word and turns the CTA's remaining work off, never its
// barriers); a last barrier keeps each CTA's shared memory alive until its
// peers have read it.  The host runs it for even rows from a 16-byte
// aligned x, so each segment starts 16-byte aligned.
template <int THREADS, int PER, int CL>
__device__ __forceinline__ void softmax_rows_cluster(
    const hexir_activation_args_t &p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ double red[THREADS / 32];
  __shared__ double part_max, part_sum;
  __shared__ __align__(8) uint64_t bar;
  double *buf = reinterpret_cast<double *>(smem_raw);
  const uint32_t cols = p.cols;
  const uint32_t rank = cluster_ctarank();
  const uint32_t seg = ((cols + CL - 1) / CL + 1u) & ~1u;
  const uint32_t c0 = min(cols, rank * seg);
  const uint32_t len = min(cols, c0 + seg) - c0;
  const uint32_t bytes = len * 8u;
  const uint64_t clusters = gridDim.x / CL;
  const uint64_t first = blockIdx.x / CL;  // the cluster's first row
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  bool live = true;  // false once a copy has run out of time
  if (threadIdx.x == 0 && first < p.rows && bytes) {
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_load(buf, p.x + first * cols + c0, bytes, &bar);
  }
  uint32_t phase = 0;
  for (uint64_t row = first; row < p.rows; row += clusters) {
    if (bytes && live) {
      const bool arrived = mbar_wait_bounded(&bar, phase, p.timeout_ns);
      phase ^= 1u;
      live = __syncthreads_and(arrived) != 0;
    }
    double v[PER];
    double m = neg_inf();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      v[i] = j < len ? buf[j] : neg_inf();
      m = v[i] > m ? v[i] : m;
    }
    m = block_reduce<THREADS>(m, red, MaxOp{});  // buf is read: free for the next row
    const uint64_t next = row + clusters;
    if (threadIdx.x == 0) {
      if (live && bytes && next < p.rows) {
        mbar_arrive_expect_tx(&bar, bytes);
        bulk_load(buf, p.x + next * cols + c0, bytes, &bar);
      }
      part_max = m;
    }
    cluster_sync();
    double rm = ld_cluster_f64(&part_max, 0);
#pragma unroll
    for (uint32_t r = 1; r < CL; ++r) {
      const double x = ld_cluster_f64(&part_max, r);
      rm = x > rm ? x : rm;
    }
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t j = threadIdx.x + i * THREADS;
      if (j < len) {
        v[i] = exp(__dsub_rn(v[i], rm));
        s = __dadd_rn(s, v[i]);
      }
    }
    s = block_reduce<THREADS>(s, red, SumOp{});
    if (threadIdx.x == 0)
      part_sum = s;
    cluster_sync();
    double rs = ld_cluster_f64(&part_sum, 0);
#pragma unroll
    for (uint32_t r = 1; r < CL; ++r)
      rs = __dadd_rn(rs, ld_cluster_f64(&part_sum, r));
    rs = __drcp_rn(rs);
    double *yr = p.out + row * cols + c0;
    if (live) {
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const uint32_t j = threadIdx.x + i * THREADS;
        if (j < len)
          __stcs(yr + j, __dmul_rn(v[i], rs));
      }
    }
  }
  cluster_sync();
}

// Rows too long for registers: maximum, sum and output each read the row
// (the second and third reads mostly from L2).
template <int THREADS>
__device__ __forceinline__ void softmax_rows_wide(
    const hexir_activation_args_t &p) {
  __shared__ double red[THREADS / 32];
  const uint32_t cols = p.cols;
  for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const double *xr = p.x + row * cols;
    double *yr = p.out + row * cols;
    double m = neg_inf();
    for (uint32_t j = threadIdx.x; j < cols; j += THREADS) {
      const double x = xr[j];
      m = x > m ? x : m;
    }
    m = block_reduce<THREADS>(m, red, MaxOp{});
    double s = 0.0;
    for (uint32_t j = threadIdx.x; j < cols; j += THREADS)
      s = __dadd_rn(s, exp(__dsub_rn(xr[j], m)));
    const double rs = __drcp_rn(block_reduce<THREADS>(s, red, SumOp{}));
    for (uint32_t j = threadIdx.x; j < cols; j += THREADS)
      __stcs(yr + j, __dmul_rn(exp(__dsub_rn(__ldcs(xr + j), m)), rs));
  }
}

}  // namespace

#define HEXIR_ACTIVATION_KERNEL(name, Op)                              \
  extern "C" __global__ void __launch_bounds__(256)                    \
      name(const hexir_activation_args_t args) {                       \
    activation_stream(args, Op{});                                     \
  }

HEXIR_ACTIVATION_KERNEL(hexir_leaky_relu_f64, LeakyReluOp)
HEXIR_ACTIVATION_KERNEL(hexir_elu_f64, EluOp)
HEXIR_ACTIVATION_KERNEL(hexir_sigmoid_f64, SigmoidOp)
HEXIR_ACTIVATION_KERNEL(hexir_tanh_f64, TanhOp)
// gelu stages its coefficient table (18 KiB) in shared memory once per
// block, then runs the same stream loop.
extern "C" __global__ void __launch_bounds__(256)
    hexir_gelu_f64(const hexir_activation_args_t args) {
  __shared__ __align__(16) double table[kGeluIntervals * kGeluRow];
  const double2 *src = reinterpret_cast<const double2 *>(&kGeluTable[0][0]);
  double2 *dst = reinterpret_cast<double2 *>(table);
  for (int i = threadIdx.x; i < kGeluIntervals * kGeluRow / 2; i += blockDim.x)
    dst[i] = src[i];
  __syncthreads();
  activation_stream(args, GeluOp{table});
}
HEXIR_ACTIVATION_KERNEL(hexir_swish_f64, SwishOp)
HEXIR_ACTIVATION_KERNEL(hexir_mish_f64, MishOp)

#undef HEXIR_ACTIVATION_KERNEL

// 256 threads = 8 rows per block.
extern "C" __global__ void __launch_bounds__(256)
    hexir_softmax_warp_f64(const hexir_activation_args_t args) {
  softmax_rows_warp<HEXIR_SOFTMAX_WARP_COLS / 32>(args);
}

extern "C" __global__ void __launch_bounds__(256, 2)
    hexir_softmax_b256_f64(const hexir_activation_args_t args) {
  softmax_rows_block<256, HEXIR_SOFTMAX_B256_COLS / 256>(args);
}

extern "C" __global__ void __launch_bounds__(512, 1)
    hexir_softmax_b512_f64(const hexir_activation_args_t args) {
  softmax_rows_block<512, HEXIR_SOFTMAX_B512_COLS / 512>(args);
}

extern "C" __global__ void __launch_bounds__(512)
    hexir_softmax_wide_f64(const hexir_activation_args_t args) {
  softmax_rows_wide<512>(args);
}

extern "C" __global__ void __launch_bounds__(256, 2)
    hexir_softmax_bulk256_f64(const hexir_activation_args_t args) {
  softmax_rows_bulk<256, HEXIR_SOFTMAX_B256_COLS / 256>(args);
}

// Long even rows over clusters of 4-8 CTAs, up to 8192 columns per CTA (the
// host sets the cluster shape at launch).
#define HEXIR_SOFTMAX_CLUSTER_KERNEL(CL)                                   \
  extern "C" __global__ void __launch_bounds__(256, 2)                     \
      hexir_softmax_cluster##CL##_f64(const hexir_activation_args_t args) { \
    softmax_rows_cluster<256, HEXIR_SOFTMAX_B256_COLS / 256, CL>(args);    \
  }
HEXIR_SOFTMAX_CLUSTER_KERNEL(4)
HEXIR_SOFTMAX_CLUSTER_KERNEL(5)
HEXIR_SOFTMAX_CLUSTER_KERNEL(6)
HEXIR_SOFTMAX_CLUSTER_KERNEL(7)
HEXIR_SOFTMAX_CLUSTER_KERNEL(8)
#undef HEXIR_SOFTMAX_CLUSTER_KERNEL

// Short rows: the same persistent bulk-prefetch blocks with fewer elements
// per thread, so more blocks (and so more row copies in flight) fit an SM.
extern "C" __global__ void __launch_bounds__(256, 5)
    hexir_softmax_bulk_s2k_f64(const hexir_activation_args_t args) {
  softmax_rows_bulk<256, HEXIR_SOFTMAX_S2K_COLS / 256>(args);
}

extern "C" __global__ void __launch_bounds__(256, 3)
    hexir_softmax_bulk_s4k_f64(const hexir_activation_args_t args) {
  softmax_rows_bulk<256, HEXIR_SOFTMAX_S4K_COLS / 256>(args);
}

extern "C" __global__ void __launch_bounds__(512, 1)
    hexir_softmax_bulk512_f64(const hexir_activation_args_t args) {
  softmax_rows_bulk<512, HEXIR_SOFTMAX_B512_COLS / 512>(args);
}
