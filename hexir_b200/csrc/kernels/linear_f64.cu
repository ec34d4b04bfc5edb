// linear_f64.cu -- f64 dense contraction c[m x n] = a[m x k] . b[k x n] on
// B200 FP64 tensor cores (DMMA, mma.sync m16n8k8 f64; tcgen05 has no f64
// kind), optionally followed by the reference relu in the epilogue.
//
// Same operation as the reference CPU kernel hexir_ref_matmul_f64
// (runtime/src/kernels/reference_kernels.c:3-13) and the generated GPU kernel
// linear_<n> (compiler/Conversion/HexirToTIR/HexirToTIR.cpp:96-170); the
// summation order over k differs (tiles of 8 on the tensor core), so results
// agree with the CPU to within f64 rounding, not bit for bit.
//
// Kernels:
//   hexir_linear_f64_tma      TMA-fed mbarrier ring, 8 DMMA warps (thread 0
//   hexir_linear_f64_tma_m64  also issues the TMA boxes), one CTA per SM;
//   hexir_linear_f64_tma_m16  CTA tiles 128x128x32 (3 stages), 64x128x32 (4)
//                             and 16x128x32 (3, two CTAs per SM) for tall,
//                             medium and skinny row counts.
//                             Needs k and n even and 16-byte aligned bases.
//   hexir_linear_f64_guarded  any shape and alignment: bounds-checked loads,
//                             64x64x16 tile, double-buffered shared memory.
//   hexir_linear_f64_splitk_reduce
//                             sums split-K partials in split order, then
//                             applies the epilogue.
//
// Shared-memory layouts (both kernels):
//   A tile [BM][BK] is held as BK/8 slabs of [BM rows][8 doubles] (64 B per
//   row).  A thread's A fragment for one k8 step is one 16-byte load.
//   B tile [BK][BN] is held as BN/16 slabs of [BK rows][16 doubles] (128 B
//   per row) with the 16-byte chunk index XORed by (row & 7) -- the TMA
//   128-byte swizzle -- so fragment loads hit 32 distinct banks.
//   Within every k8 step the MMA's k slot s maps to physical k 2s (s < 4) and
//   2(s-4)+1 (s >= 4), and within every 16-column block MMA tile j column nn
//   maps to physical column 2nn + j.  Both permutations are applied to A and
//   B alike, so the product is unchanged; they make every fragment a 16-byte
//   load and every output row segment of a thread 4 contiguous doubles.

#include "common.cuh"

namespace hexir {


// Grouped raster: group_m row-tiles share each sweep over the column tiles,
// so concurrently running CTAs reuse the same A and B panels from L2.
__device__ __forceinline__ void tile_of(uint32_t linear, uint32_t tiles_m,
                                        uint32_t tiles_n, uint32_t group_m,
                                        uint32_t &tm, uint32_t &tn) {
  const uint32_t per_group = group_m * tiles_n;
  const uint32_t group = linear / per_group;
  const uint32_t first_m = group * group_m;
  const uint32_t rows = min(group_m, tiles_m - first_m);
  const uint32_t in_group = linear - group * per_group;
  tm = first_m + in_group % rows;
  tn = in_group / rows;
}

// One k8 step of a warp tile of MI m16-tiles by NP 16-column blocks.
//   a_slab   shared address of the [rows][8] A slab holding this k8 step
//   a_row    first tile row of this warp
//   b_slab   shared address of the warp's first [rows][16] B slab
//   b_stride bytes between consecutive B slabs
//   k_row    row of this k8 step inside the B slabs (a multiple of 8)
template <int MI, int NP>
__device__ __forceinline__ void dmma_k8_step(double (&acc)[MI][2 * NP][4],
                                             uint32_t a_slab, uint32_t a_row,
                                             uint32_t b_slab,
                                             uint32_t b_stride, uint32_t k_row,
                                             uint32_t g, uint32_t t) {
  double2 alo[MI], ahi[MI];
#pragma unroll
  for (int mi = 0; mi < MI; ++mi) {
    const uint32_t r = a_row + mi * 16 + g;
    alo[mi] = lds128(a_slab + r * 64 + t * 16);
    ahi[mi] = lds128(a_slab + (r + 8) * 64 + t * 16);
  }
  double2 bk0[NP], bk1[NP];
  const uint32_t r0 = k_row + 2 * t, r1 = r0 + 1;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const uint32_t base = b_slab + p * b_stride;
    bk0[p] = lds128(base + r0 * 128 + ((g ^ (r0 & 7)) << 4));
    bk1[p] = lds128(base + r1 * 128 + ((g ^ (r1 & 7)) << 4));
  }
#pragma unroll
  for (int mi = 0; mi < MI; ++mi) {
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      dmma_16x8x8(acc[mi][2 * p], alo[mi].x, ahi[mi].x, alo[mi].y, ahi[mi].y,
                  bk0[p].x, bk1[p].x);
      dmma_16x8x8(acc[mi][2 * p + 1], alo[mi].x, ahi[mi].x, alo[mi].y,
                  ahi[mi].y, bk0[p].y, bk1[p].y);
    }
  }
}

// Write a warp tile.  Row r of m16-tile mi holds, in this thread, the four
// consecutive columns col..col+3 = (tile 2p).d0, (2p+1).d0, (2p).d1, (2p+1).d1;
// row r+8 the same with d2, d3.
template <int MI, int NP, bool VEC>
__device__ __forceinline__ void store_warp_tile(
    const double (&acc)[MI][2 * NP][4], double *__restrict__ c, uint32_t m,
    uint32_t n, uint32_t row0, uint32_t col0, bool relu, uint32_t g,
    uint32_t t, bool vec4 = false, const double *__restrict__ addend = nullptr,
    bool stream = false) {
#pragma unroll
  for (int mi = 0; mi < MI; ++mi) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t row = row0 + mi * 16 + g + half * 8;
      if (row >= m)
        continue;
      double *crow = c + (size_t)row * n;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint32_t col = col0 + p * 16 + 4 * t;
        double v[4] = {acc[mi][2 * p][2 * half], acc[mi][2 * p + 1][2 * half],
                       acc[mi][2 * p][2 * half + 1],
                       acc[mi][2 * p + 1][2 * half + 1]};
        if (addend) {
          // The fused add: the same rounding as adding the stored product.
          const double *arow = addend + (size_t)row * n;
          double b[4] = {0.0, 0.0, 0.0, 0.0};
          if (VEC && vec4) {
            if (col < n)
              ldg256(arow + col, b);
          } else if (VEC) {
            if (col < n) {
              const double2 x = *reinterpret_cast<const double2 *>(arow + col);
              b[0] = x.x;
              b[1] = x.y;
            }
            if (col + 2 < n) {
              const double2 x = *reinterpret_cast<const double2 *>(arow + col + 2);
              b[2] = x.x;
              b[3] = x.y;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (col + q < n)
                b[q] = arow[col + q];
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            v[q] = __dadd_rn(v[q], b[q]);
        }
        if (relu) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            v[q] = relu_ref(v[q]);
        }
        if (VEC && vec4) {
          // n % 4 == 0 and rows 32-byte aligned: quads never straddle n.
          if (col < n) {
            if (stream)
              stg256_cs(crow + col, v[0], v[1], v[2], v[3]);
            else
              stg256(crow + col, v[0], v[1], v[2], v[3]);
          }
        } else if (VEC) {
          // n is even and the base 16-byte aligned: pairs never straddle n.
          double2 *q = reinterpret_cast<double2 *>(crow + col);
          if (col < n) {
            if (stream)
              __stcs(q, make_double2(v[0], v[1]));
            else
              *q = make_double2(v[0], v[1]);
          }
          if (col + 2 < n) {
            if (stream)
              __stcs(q + 1, make_double2(v[2], v[3]));
            else
              q[1] = make_double2(v[2], v[3]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (col + q < n)
              crow[col + q] = v[q];
        }
      }
    }
  }
}

// Start a warp tile's sums from c_in: the inverse of store_warp_tile's
// mapping (elements outside m x n stay 0 and are never stored).
template <int MI, int NP, bool VEC>
__device__ __forceinline__ void load_warp_tile(
    double (&acc)[MI][2 * NP][4], const double *__restrict__ c_in, uint32_t m,
    uint32_t n, uint32_t row0, uint32_t col0, uint32_t g, uint32_t t,
    bool vec4 = false) {
#pragma unroll
  for (int mi = 0; mi < MI; ++mi) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t row = row0 + mi * 16 + g + half * 8;
      if (row >= m)
        continue;
      const double *crow = c_in + (size_t)row * n;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint32_t col = col0 + p * 16 + 4 * t;
        double v[4] = {0.0, 0.0, 0.0, 0.0};
        if (VEC && vec4) {
          if (col < n)
            ldg256(crow + col, v);
        } else if (VEC) {
          if (col < n) {
            const double2 x = *reinterpret_cast<const double2 *>(crow + col);
            v[0] = x.x;
            v[1] = x.y;
          }
          if (col + 2 < n) {
            const double2 x = *reinterpret_cast<const double2 *>(crow + col + 2);
            v[2] = x.x;
            v[3] = x.y;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (col + q < n)
              v[q] = crow[col + q];
        }
        acc[mi][2 * p][2 * half] = v[0];
        acc[mi][2 * p + 1][2 * half] = v[1];
        acc[mi][2 * p][2 * half + 1] = v[2];
        acc[mi][2 * p + 1][2 * half + 1] = v[3];
      }
    }
  }
}

}  // namespace hexir

using namespace hexir;

namespace hexir {

// Tile configurations of the TMA pipeline.  All use 8 DMMA warps (256
// threads, one CTA per SM); thread 0 also issues the TMA boxes.
//   BM x BN x BK  CTA tile; STAGES smem ring depth
//   WARPS_M x WARPS_N  warp grid; warp tile (BM/WARPS_M) x (BN/WARPS_N)
template <int BM_, int BN_, int BK_, int STAGES_, int WARPS_M_>
struct TmaTile {
  static constexpr int BM = BM_, BN = BN_, BK = BK_, STAGES = STAGES_;
  static constexpr int WARPS_M = WARPS_M_, WARPS_N = 8 / WARPS_M_;
  static constexpr int WTM = BM / WARPS_M, WTN = BN / WARPS_N;  // warp tile
  static constexpr int MI = WTM / 16, NP = WTN / 16;
  static constexpr int A_SLAB = BM * 8, B_SLAB = BK * 16;  // doubles per box
  static constexpr int A_STAGE = BM * BK, B_STAGE = BK * BN;
  static constexpr uint32_t STAGE_BYTES = (A_STAGE + B_STAGE) * 8;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(MI >= 1 && NP >= 1 && WTM % 16 == 0 && WTN % 16 == 0,
                "warp tile must be a multiple of 16 x 16");
  static_assert((B_SLAB * 8) % 1024 == 0 && (A_STAGE * 8) % 1024 == 0,
                "slabs must keep the 1024-B swizzle alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

using Tile128 = TmaTile<HEXIR_LINEAR_BM, HEXIR_LINEAR_BN, HEXIR_LINEAR_BK,
                        HEXIR_LINEAR_STAGES, 2>;
using Tile64 = TmaTile<64, 128, 32, 4, 2>;
using Tile16 = TmaTile<16, 128, 32, 3, 1>;
static_assert(Tile128::SMEM_BYTES == HEXIR_LINEAR_SMEM_BYTES, "smem");
static_assert(Tile64::SMEM_BYTES == HEXIR_LINEAR_M64_SMEM_BYTES, "smem");
static_assert(Tile16::SMEM_BYTES == HEXIR_LINEAR_M16_SMEM_BYTES, "smem");

template <class T>
__device__ __forceinline__ void linear_tma_body(const CUtensorMap *map_a,
                                                const CUtensorMap *map_b,
                                                const hexir_linear_args_t &args) {
  constexpr int BM = T::BM, BN = T::BN, BK = T::BK, STAGES = T::STAGES;
  constexpr int MI = T::MI, NP = T::NP;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align the ring to the 1024-byte swizzle atom.
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  double *sa = reinterpret_cast<double *>(smem);
  double *sb = sa + STAGES * T::A_STAGE;
  uint64_t *full = reinterpret_cast<uint64_t *>(sb + STAGES * T::B_STAGE);
  uint64_t *empty = full + STAGES;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool issuer = threadIdx.x == 0;

  uint32_t tm, tn;
  tile_of(blockIdx.x, args.tiles_m, args.tiles_n, args.group_m, tm, tn);
  const uint32_t split = blockIdx.y;
  const uint32_t kt_begin = split * args.k_tiles_per_split;
  const uint32_t kt_end = min(args.k_tiles, kt_begin + args.k_tiles_per_split);
  const int32_t nk = kt_end > kt_begin ? (int32_t)(kt_end - kt_begin) : 0;
  const uint32_t m0 = tm * BM, n0 = tn * BN;

  if (issuer) {
    prefetch_tensormap(map_a);
    prefetch_tensormap(map_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HEXIR_LINEAR_CONSUMER_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // Thread 0 arms stage s for k-tile i and issues its TMA boxes: BK/8 A boxes
  // of [BM][8] and BN/16 B boxes of [BK][16] (128-byte swizzled).
  auto issue = [&](int32_t i) {
    const int s = i % STAGES;
    mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
    const int32_t k0 = (int32_t)((kt_begin + i) * BK);
    double *as = sa + s * T::A_STAGE;
    double *bs = sb + s * T::B_STAGE;
#pragma unroll
    for (int j = 0; j < BK / 8; ++j)
      tma_load_2d(as + j * T::A_SLAB, map_a, k0 + j * 8, (int32_t)m0, &full[s]);
#pragma unroll
    for (int j = 0; j < BN / 16; ++j)
      tma_load_2d(bs + j * T::B_SLAB, map_b, (int32_t)(n0 + j * 16), k0,
                  &full[s]);
  };
  int32_t issued = 0;
  if (issuer) {
    for (; issued < nk && issued < STAGES; ++issued)
      issue(issued);
  }

  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t wm = warp / T::WARPS_N, wn = warp % T::WARPS_N;
  double acc[MI][2 * NP][4];
#pragma unroll
  for (int i = 0; i < MI; ++i)
#pragma unroll
    for (int j = 0; j < 2 * NP; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        acc[i][j][q] = 0.0;
  const bool vec4 = (args.epilogue & HEXIR_EPILOGUE_VEC4) != 0;
  if (args.c_in)
    load_warp_tile<MI, NP, true>(acc, args.c_in, args.m, args.n,
                                 m0 + wm * T::WTM, n0 + wn * T::WTN, g, t, vec4);

  const uint32_t sa_addr = smem_addr(sa), sb_addr = smem_addr(sb);
  bool ok = true;
  for (int32_t i = 0; i < nk; ++i) {
    const int s = i % STAGES;
    const uint32_t use = (uint32_t)i / STAGES;
    if (!mbar_wait_bounded(&full[s], use & 1u, args.timeout_ns)) {
      ok = false;
      break;
    }
    const uint32_t a_stage = sa_addr + s * T::A_STAGE * 8;
    const uint32_t b_stage =
        sb_addr + s * T::B_STAGE * 8 + (wn * NP) * T::B_SLAB * 8;
#pragma unroll
    for (int kk = 0; kk < BK / 8; ++kk)
      dmma_k8_step<MI, NP>(acc, a_stage + kk * T::A_SLAB * 8, wm * T::WTM,
                           b_stage, T::B_SLAB * 8, kk * 8, g, t);
    __syncwarp();
    if (lane == 0)
      mbar_arrive(&empty[s]);
    // Refill stage s with k-tile i + STAGES once all 8 warps released it.
    if (issuer && issued < nk) {
      if (!mbar_wait_bounded(&empty[s], use & 1u, args.timeout_ns)) {
        ok = false;
        break;
      }
      issue(issued++);
    }
    // Reconverge warp 0 before the next iteration's warp-wide DMMAs.
    __syncwarp();
  }

  if (issuer) {
    // Nothing may still be writing this CTA's shared memory when it exits.
    // Stage s was armed ceil((issued - s) / STAGES) times; wait for the phase
    // of its last arm.  After a normal run these return at once.
#pragma unroll
    for (int s = 0; s < STAGES; ++s)
      if (issued > s) {
        const uint32_t uses = (uint32_t)(issued - s + STAGES - 1) / STAGES;
        mbar_wait_bounded(&full[s], (uses - 1) & 1u, args.timeout_ns);
      }
  }
  if (!ok)
    return;

  double *dst = args.c;
  bool relu = (args.epilogue & HEXIR_EPILOGUE_RELU) != 0;
  const double *addend =
      (args.epilogue & HEXIR_EPILOGUE_ADD) ? args.addend : nullptr;
  if (args.split_k > 1) {
    dst += (size_t)split * args.m * args.n;
    relu = false;
    addend = nullptr;
  }
  store_warp_tile<MI, NP, true>(
      acc, dst, args.m, args.n, m0 + wm * T::WTM, n0 + wn * T::WTN, relu, g, t,
      vec4, addend,
      args.split_k == 1 && (args.epilogue & HEXIR_EPILOGUE_STREAM) != 0);
  if (args.split_k == 1 && (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE))
    __threadfence_system();
}

// The k-tile steps of one CTA of a stream-K launch, in the order it runs
// them: its data-parallel tiles whole, then its run of stream-K units.  The
// producer and the consumers each walk them with a Cursor, which advances by
// increments (no division per step: the per-k-tile budget of the DMMA loop
// has no issue slots to spare).
struct SkSteps {
  uint32_t c, grid, dp_tiles, k_tiles, dp_steps, u0, n_steps;
  __device__ __forceinline__ SkSteps(const hexir_linear_args_t &args) {
    c = blockIdx.x;
    grid = gridDim.x;
    dp_tiles = args.sk_dp_tiles;
    k_tiles = args.k_tiles;
    const uint32_t tiles = args.tiles_m * args.tiles_n;
    const uint32_t my_dp = dp_tiles > c ? (dp_tiles - c - 1) / grid + 1 : 0;
    dp_steps = my_dp * k_tiles;
    const uint32_t sk_total = (tiles - dp_tiles) * k_tiles;
    u0 = min(c * args.sk_units, sk_total);
    const uint32_t u1 = min(u0 + args.sk_units, sk_total);
    n_steps = dp_steps + (u1 - u0);
  }
  __device__ __forceinline__ uint32_t first_sk_tile() const {
    return dp_tiles + u0 / k_tiles;
  }
  // Position (tile, kt) of step i, advanced one step at a time.
  struct Cursor {
    uint32_t i, tile, kt;
  };
  __device__ __forceinline__ Cursor begin() const {
    Cursor p;
    p.i = 0;
    if (dp_steps) {
      p.tile = c;
      p.kt = 0;
    } else {
      p.tile = first_sk_tile();
      p.kt = u0 % k_tiles;
    }
    return p;
  }
  __device__ __forceinline__ void next(Cursor &p) const {
    ++p.i;
    if (p.i == dp_steps) {
      p.tile = first_sk_tile();
      p.kt = u0 % k_tiles;
    } else if (++p.kt == k_tiles) {
      p.kt = 0;
      p.tile += p.i < dp_steps ? grid : 1u;
    }
  }
};

template <class T>
__device__ __forceinline__ void linear_tma_sk_body(
    const CUtensorMap *map_a, const CUtensorMap *map_b,
    const hexir_linear_args_t &args) {
  constexpr int BM = T::BM, BN = T::BN, BK = T::BK, STAGES = T::STAGES;
  constexpr int MI = T::MI, NP = T::NP;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  double *sa = reinterpret_cast<double *>(smem);
  double *sb = sa + STAGES * T::A_STAGE;
  uint64_t *full = reinterpret_cast<uint64_t *>(sb + STAGES * T::B_STAGE);
  uint64_t *empty = full + STAGES;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool issuer = threadIdx.x == 0;
  const SkSteps steps(args);
  const int32_t nk = (int32_t)steps.n_steps;

  if (issuer) {
    prefetch_tensormap(map_a);
    prefetch_tensormap(map_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HEXIR_LINEAR_CONSUMER_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // The producer's cursor and the row / column of its current tile.
  SkSteps::Cursor prod = steps.begin();
  uint32_t prod_tile = ~0u, ptm = 0, ptn = 0;
  auto issue = [&](int32_t i) {
    const int s = i % STAGES;
    if (prod.tile != prod_tile) {
      prod_tile = prod.tile;
      tile_of(prod_tile, args.tiles_m, args.tiles_n, args.group_m, ptm, ptn);
    }
    const uint32_t tm = ptm, tn = ptn, kt = prod.kt;
    steps.next(prod);
    mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
    const int32_t k0 = (int32_t)(kt * BK);
    double *as = sa + s * T::A_STAGE;
    double *bs = sb + s * T::B_STAGE;
#pragma unroll
    for (int j = 0; j < BK / 8; ++j)
      tma_load_2d(as + j * T::A_SLAB, map_a, k0 + j * 8, (int32_t)(tm * BM),
                  &full[s]);
#pragma unroll
    for (int j = 0; j < BN / 16; ++j)
      tma_load_2d(bs + j * T::B_SLAB, map_b, (int32_t)(tn * BN + j * 16), k0,
                  &full[s]);
  };
  int32_t issued = 0;
  if (issuer) {
    for (; issued < nk && issued < STAGES; ++issued)
      issue(issued);
  }

  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t wm = warp / T::WARPS_N, wn = warp % T::WARPS_N;
  const bool relu = (args.epilogue & HEXIR_EPILOGUE_RELU) != 0;
  const bool vec4 = (args.epilogue & HEXIR_EPILOGUE_VEC4) != 0;
  const double *addend =
      (args.epilogue & HEXIR_EPILOGUE_ADD) ? args.addend : nullptr;
  double acc[MI][2 * NP][4];
  const uint32_t sa_addr = smem_addr(sa), sb_addr = smem_addr(sb);
  bool ok = true;
  // Segments: a whole data-parallel tile, or the part of a stream-K tile in
  // this CTA's run.  The inner loop over a segment's k-tiles is the
  // data-parallel kernel's loop; the epilogue follows it.
  int32_t i = 0;
  uint32_t tile = steps.dp_steps ? steps.c : steps.first_sk_tile();
  uint32_t kt0 = steps.dp_steps ? 0u : steps.u0 % steps.k_tiles;
  while (i < nk) {
    const int32_t seg_len = min((int32_t)(args.k_tiles - kt0), nk - i);
#pragma unroll
    for (int a = 0; a < MI; ++a)
#pragma unroll
      for (int b = 0; b < 2 * NP; ++b)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          acc[a][b][q] = 0.0;
    for (int32_t j = 0; j < seg_len; ++j, ++i) {
      const int s = i % STAGES;
      const uint32_t use = (uint32_t)i / STAGES;
      if (!mbar_wait_bounded(&full[s], use & 1u, args.timeout_ns)) {
        ok = false;
        break;
      }
      const uint32_t a_stage = sa_addr + s * T::A_STAGE * 8;
      const uint32_t b_stage =
          sb_addr + s * T::B_STAGE * 8 + (wn * NP) * T::B_SLAB * 8;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk)
        dmma_k8_step<MI, NP>(acc, a_stage + kk * T::A_SLAB * 8, wm * T::WTM,
                             b_stage, T::B_SLAB * 8, kk * 8, g, t);
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&empty[s]);
      if (issuer && issued < nk) {
        if (!mbar_wait_bounded(&empty[s], use & 1u, args.timeout_ns)) {
          ok = false;
          break;
        }
        issue(issued++);
      }
      __syncwarp();
    }
    if (!ok)
      break;
    uint32_t tm, tn;
    tile_of(tile, args.tiles_m, args.tiles_n, args.group_m, tm, tn);
    if (kt0 == 0 && (uint32_t)seg_len == args.k_tiles) {
      store_warp_tile<MI, NP, true>(acc, args.c, args.m, args.n,
                                    tm * BM + wm * T::WTM, tn * BN + wn * T::WTN,
                                    relu, g, t, vec4, addend);
    } else {
      const uint32_t slot =
          2 * steps.c + (tile == steps.first_sk_tile() ? 0u : 1u);
      store_warp_tile<MI, NP, true>(acc, args.sk_partials + (size_t)slot * BM * BN,
                                    BM, BN, wm * T::WTM, wn * T::WTN, false, g,
                                    t, true, nullptr);
    }
    // The next segment: the next data-parallel tile, the start of the
    // stream-K run, or the next stream-K tile.
    if ((uint32_t)i == steps.dp_steps) {
      tile = steps.first_sk_tile();
      kt0 = steps.u0 % steps.k_tiles;
    } else {
      tile += (uint32_t)i < steps.dp_steps ? steps.grid : 1u;
      kt0 = 0;
    }
  }

  if (issuer) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s)
      if (issued > s) {
        const uint32_t uses = (uint32_t)(issued - s + STAGES - 1) / STAGES;
        mbar_wait_bounded(&full[s], (uses - 1) & 1u, args.timeout_ns);
      }
  }
  if (ok && (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE))
    __threadfence_system();
}

}  // namespace hexir

// 128 x 128 x 32 CTA tile: square and tall shapes (warp tile 64 x 32).
extern "C" __global__ void __launch_bounds__(HEXIR_LINEAR_THREADS, 1)
    hexir_linear_f64_tma(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b,
                         const hexir_linear_args_t args) {
  linear_tma_body<Tile128>(&map_a, &map_b, args);
}

// The 128 x 128 x 32 pipeline as a persistent stream-K launch (one CTA per
// SM, see SkSteps): shapes with too few tiles to fill whole waves.
extern "C" __global__ void __launch_bounds__(HEXIR_LINEAR_THREADS, 1)
    hexir_linear_f64_tma_sk(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b,
                            const hexir_linear_args_t args) {
  linear_tma_sk_body<Tile128>(&map_a, &map_b, args);
}

// Completes the stream-K tiles whose k units were split over CTAs: one CTA
// per such tile sums the partial tiles in CTA order (the order of k), then
// applies the epilogue (addend, relu).  Tiles owned by one CTA were stored by
// it and are skipped.
extern "C" __global__ void __launch_bounds__(256)
    hexir_linear_f64_sk_fixup(const hexir_linear_args_t args) {
  constexpr uint32_t BM = HEXIR_LINEAR_BM, BN = HEXIR_LINEAR_BN;
  const uint32_t tile = args.sk_dp_tiles + blockIdx.x;
  const uint32_t k_tiles = args.k_tiles, U = args.sk_units;
  const uint32_t t0 = blockIdx.x * k_tiles;  // first unit of the tile
  const uint32_t c0 = t0 / U, c1 = (t0 + k_tiles - 1) / U;
  if (c0 == c1)
    return;
  uint32_t tm, tn;
  tile_of(tile, args.tiles_m, args.tiles_n, args.group_m, tm, tn);
  const bool relu = (args.epilogue & HEXIR_EPILOGUE_RELU) != 0;
  const bool add = (args.epilogue & HEXIR_EPILOGUE_ADD) != 0;
  for (uint32_t e = threadIdx.x; e < BM * BN; e += blockDim.x) {
    const uint32_t r = e / BN, col = e % BN;
    const uint32_t row = tm * BM + r, gcol = tn * BN + col;
    if (row >= args.m || gcol >= args.n)
      continue;
    double s = 0.0;
    for (uint32_t c = c0; c <= c1; ++c) {
      // The CTA's run starts in this tile: its first-tile slot.
      const uint32_t first = args.sk_dp_tiles + (c * U) / k_tiles;
      const uint32_t slot = 2 * c + (tile == first ? 0u : 1u);
      s = __dadd_rn(s, args.sk_partials[(size_t)slot * BM * BN + e]);
    }
    const size_t idx = (size_t)row * args.n + gcol;
    if (add)
      s = __dadd_rn(s, args.addend[idx]);
    args.c[idx] = relu ? relu_ref(s) : s;
  }
  if (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE)
    __threadfence_system();
}

// 64 x 128 x 32, 4 stages: 17..64 rows (warp tile 32 x 32).
extern "C" __global__ void __launch_bounds__(HEXIR_LINEAR_THREADS, 1)
    hexir_linear_f64_tma_m64(const __grid_constant__ CUtensorMap map_a,
                             const __grid_constant__ CUtensorMap map_b,
                             const hexir_linear_args_t args) {
  linear_tma_body<Tile64>(&map_a, &map_b, args);
}

// 16 x 128 x 32, 3 stages, two CTAs per SM: up to 16 rows, where the weight
// stream is the whole cost (warp tile 16 x 16, one m16 DMMA row block).  Two
// resident CTAs hide each other's pipeline fill; measured 6.4 TB/s on the
// weight read at m = 1, against 4.4-4.8 TB/s for one 6-stage CTA per SM.
extern "C" __global__ void __launch_bounds__(HEXIR_LINEAR_THREADS, 2)
    hexir_linear_f64_tma_m16(const __grid_constant__ CUtensorMap map_a,
                             const __grid_constant__ CUtensorMap map_b,
                             const hexir_linear_args_t args) {
  linear_tma_body<Tile16>(&map_a, &map_b, args);
}

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
