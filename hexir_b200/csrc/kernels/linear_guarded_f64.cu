// linear_guarded_f64.cu -- the f64 linear for shapes the TMA kernels cannot
// describe, and the split-K reduction.
//
// Same operation as the reference CPU kernel hexir_ref_matmul_f64
// (runtime/src/kernels/reference_kernels.c:3-13), on the DMMA tiles of
// linear_tiles.cuh.  Kernels:
//   hexir_linear_f64_guarded  any shape and alignment: bounds-checked loads,
//                             64x64x16 tile, double-buffered shared memory.
//   hexir_linear_f64_splitk_reduce
//                             sums split-K partials in split order, then
//                             applies the epilogue.
// Neither waits on a barrier other than __syncthreads, so neither sets the
// device error word.  This file is also the whole device code of the
// no-alloc entry point (runtime/matmul_noalloc.cu).

#include "linear_tiles.cuh"

using namespace hexir;

// Guarded variant: every global load is bounds checked, so any m, n, k and
// any 8-byte alignment works (odd k or n, 1x1x1, row shards at odd offsets).
extern "C" __global__ void __launch_bounds__(HEXIR_LINEAR_G_THREADS)
    hexir_linear_f64_guarded(const hexir_linear_args_t args) {
  constexpr int BM = HEXIR_LINEAR_G_BM, BN = HEXIR_LINEAR_G_BN,
                BK = HEXIR_LINEAR_G_BK;
  constexpr int A_SLAB = BM * 8, B_SLAB = BK * 16;
  constexpr int A_STAGE = BM * BK, B_STAGE = BK * BN;
  constexpr int PER_THREAD_A = A_STAGE / HEXIR_LINEAR_G_THREADS;  // 8
  constexpr int PER_THREAD_B = B_STAGE / HEXIR_LINEAR_G_THREADS;  // 8
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  double *sa = reinterpret_cast<double *>(smem_raw);
  double *sb = sa + 2 * A_STAGE;

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t wm = warp >> 1, wn = warp & 1;  // warp tile 32 x 32

  uint32_t tm, tn;
  tile_of(blockIdx.x, args.tiles_m, args.tiles_n, args.group_m, tm, tn);
  const uint32_t split = blockIdx.y;
  const uint32_t k_tiles = (args.k + BK - 1) / BK;
  const uint32_t kt_begin = split * args.k_tiles_per_split;
  const uint32_t kt_end = min(k_tiles, kt_begin + args.k_tiles_per_split);
  const uint32_t m0 = tm * BM, n0 = tn * BN;
  const uint32_t m = args.m, n = args.n, k = args.k;
  if (args.split_k > 1)
    griddep_launch_dependents();  // the reduction may start launching
  const size_t lda = args.lda ? args.lda : k;
  const double *__restrict__ a = args.a;
  const double *__restrict__ b = args.b;

  double ra[PER_THREAD_A], rb[PER_THREAD_B];
  auto load_tile = [&](uint32_t kt) {
    const uint32_t k0 = kt * BK;
#pragma unroll
    for (int i = 0; i < PER_THREAD_A; ++i) {
      const uint32_t e = tid + i * HEXIR_LINEAR_G_THREADS;
      const uint32_t row = e / BK, kc = e % BK;
      const uint32_t gr = m0 + row, gk = k0 + kc;
      ra[i] = (gr < m && gk < k) ? a[(size_t)gr * lda + gk] : 0.0;
    }
#pragma unroll
    for (int i = 0; i < PER_THREAD_B; ++i) {
      const uint32_t e = tid + i * HEXIR_LINEAR_G_THREADS;
      const uint32_t kr = e / BN, col = e % BN;
      const uint32_t gk = k0 + kr, gc = n0 + col;
      rb[i] = (gk < k && gc < n) ? b[(size_t)gk * n + gc] : 0.0;
    }
  };
  auto store_tile = [&](int buf) {
    double *as = sa + buf * A_STAGE;
    double *bs = sb + buf * B_STAGE;
#pragma unroll
    for (int i = 0; i < PER_THREAD_A; ++i) {
      const uint32_t e = tid + i * HEXIR_LINEAR_G_THREADS;
      const uint32_t row = e / BK, kc = e % BK;
      as[(kc >> 3) * A_SLAB + row * 8 + (kc & 7)] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < PER_THREAD_B; ++i) {
      const uint32_t e = tid + i * HEXIR_LINEAR_G_THREADS;
      const uint32_t kr = e / BN, col = e % BN;
      const uint32_t chunk = ((col & 15) >> 1) ^ (kr & 7);
      bs[(col >> 4) * B_SLAB + kr * 16 + chunk * 2 + (col & 1)] = rb[i];
    }
  };

  double acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        acc[i][j][q] = 0.0;
  if (args.c_in)
    load_warp_tile<2, 2, false>(acc, args.c_in, m, n, m0 + wm * 32,
                                n0 + wn * 32, g, t);

  if (kt_begin < kt_end) {
    load_tile(kt_begin);
    store_tile(0);
    __syncthreads();
    const uint32_t sa_addr = smem_addr(sa), sb_addr = smem_addr(sb);
    for (uint32_t kt = kt_begin; kt < kt_end; ++kt) {
      const int buf = (kt - kt_begin) & 1;
      const bool more = kt + 1 < kt_end;
      if (more)
        load_tile(kt + 1);
      const uint32_t a_stage = sa_addr + buf * A_STAGE * 8;
      const uint32_t b_stage = sb_addr + buf * B_STAGE * 8 + wn * 2 * B_SLAB * 8;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk)
        dmma_k8_step<2, 2>(acc, a_stage + kk * A_SLAB * 8, wm * 32, b_stage,
                           B_SLAB * 8, kk * 8, g, t);
      if (more)
        store_tile(buf ^ 1);
      __syncthreads();
    }
  }

  double *dst = args.c;
  bool relu = (args.epilogue & HEXIR_EPILOGUE_RELU) != 0;
  const double *addend =
      (args.epilogue & HEXIR_EPILOGUE_ADD) ? args.addend : nullptr;
  if (args.split_k > 1) {
    dst += (size_t)split * m * n;
    relu = false;
    addend = nullptr;
  }
  store_warp_tile<2, 2, false>(acc, dst, m, n, m0 + wm * 32, n0 + wn * 32,
                               relu, g, t, false, addend);
  if (args.split_k == 1 && (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE))
    __threadfence_system();
}

// c[i] = epilogue(sum over s in 0..split-1 of partials[s][i]), summed in
// split order so the result does not depend on scheduling; the epilogue adds
// addend[i] (HEXIR_EPILOGUE_ADD), then applies the relu.
extern "C" __global__ void __launch_bounds__(256)
    hexir_linear_f64_splitk_reduce(const hexir_reduce_args_t args) {
  griddep_wait();  // the split launch's partial sums
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const bool relu = (args.epilogue & HEXIR_EPILOGUE_RELU) != 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
       i < args.count; i += stride) {
    double s = 0.0;
    for (uint32_t p = 0; p < args.split; ++p)
      s = __dadd_rn(s, args.partials[(size_t)p * args.count + i]);
    if (args.epilogue & HEXIR_EPILOGUE_ADD)
      s = __dadd_rn(s, args.addend[i]);
    args.c[i] = relu ? relu_ref(s) : s;
  }
  if (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE)
    __threadfence_system();
}
