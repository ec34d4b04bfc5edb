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
//   hexir_linear_f64_tma      TMA-fed mbarrier ring, 8 DMMA warps (the warp
//   hexir_linear_f64_tma_m64  that releases a stage last refills it), one
//                             CTA per SM;
//   hexir_linear_f64_tma_m16  CTA tiles 128x128x32 (3 stages), 64x128x32 (4)
//                             and 16x128x32 (3, two CTAs per SM) for tall,
//                             medium and skinny row counts.
//                             Needs k and n even and 16-byte aligned bases.
//   hexir_linear_f64_tma_sk   the 128x128x32 pipeline as a persistent
//   hexir_linear_f64_sk_fixup stream-K launch, and the kernel that sums the
//                             tiles whose k range was split over CTAs.
//   (hexir_linear_f64_guarded and hexir_linear_f64_splitk_reduce, which
//   need no TMA, are in linear_guarded_f64.cu.)

#include "linear_tiles.cuh"

using namespace hexir;

namespace hexir {

// Tile configurations of the TMA pipeline.  All use 8 DMMA warps (256
// threads, one CTA per SM); thread 0 issues the first STAGES k-tiles' TMA
// boxes and the warp that releases a stage last issues its refill.  (A
// ninth, producer-only warp does not fit: three warps on one SM
// sub-partition cap a thread at 168 registers, and the 128-row tile needs
// 194.)
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
  // Per stage, how many warp releases it has seen (8 per use), and how many
  // times the stages were armed in all.
  uint32_t *released = reinterpret_cast<uint32_t *>(full + STAGES);
  uint32_t *armed = released + STAGES;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool issuer = threadIdx.x == 0;

  uint32_t tm, tn;
  tile_of(blockIdx.x, args.tiles_m, args.tiles_n, args.group_m, tm, tn);
  const uint32_t split = blockIdx.y;
  const uint32_t kt_begin = split * args.k_tiles_per_split;
  const uint32_t kt_end = min(args.k_tiles, kt_begin + args.k_tiles_per_split);
  const int32_t nk = kt_end > kt_begin ? (int32_t)(kt_end - kt_begin) : 0;
  const uint32_t m0 = tm * BM, n0 = tn * BN;
  // A split launch is followed by the reduction, which may start launching
  // once every CTA of this grid has started (the last wave).
  if (args.split_k > 1)
    griddep_launch_dependents();

  if (issuer) {
    prefetch_tensormap(map_a);
    prefetch_tensormap(map_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      released[s] = 0u;
    }
    *armed = (uint32_t)min(nk, (int32_t)STAGES);
    fence_mbar_init();
  }
  __syncthreads();

  // Arm stage s for k-tile i and issue its TMA boxes: BK/8 A boxes of
  // [BM][8] and BN/16 B boxes of [BK][16] (128-byte swizzled).  Thread 0
  // issues the first STAGES k-tiles; after that the warp that releases a
  // stage last refills it, so no warp waits for another to finish a k-tile.
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
  if (issuer) {
    for (int32_t i = 0; i < nk && i < STAGES; ++i)
      issue(i);
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
    // The warp leaves together if any lane's wait ran out: the DMMAs below
    // are warp-wide.
    if (!__all_sync(0xffffffffu,
                    mbar_wait_bounded(&full[s], use & 1u, args.timeout_ns))) {
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
    // Release stage s.  Every warp releases each use of it once, and no
    // warp can release the next use before the refill lands, so the 8th
    // release of a use is the last: that warp refills the stage with
    // k-tile i + STAGES (its acquire orders the refill after every warp's
    // reads of the stage).
    if (lane == 0) {
      const uint32_t before = atom_add_acq_rel_cta(&released[s], 1u);
      if (before % HEXIR_LINEAR_CONSUMER_WARPS ==
              HEXIR_LINEAR_CONSUMER_WARPS - 1 &&
          i + STAGES < nk) {
        issue(i + STAGES);
        atomicAdd(armed, 1u);
      }
    }
    __syncwarp();
  }

  double *dst = args.c;
  bool relu = (args.epilogue & HEXIR_EPILOGUE_RELU) != 0;
  const double *addend =
      (args.epilogue & HEXIR_EPILOGUE_ADD) ? args.addend : nullptr;
  if (args.split_k > 1) {
    dst += (size_t)split * args.m * args.n;
    relu = false;
    addend = nullptr;
  }
  if (ok) {
    store_warp_tile<MI, NP, true>(
        acc, dst, args.m, args.n, m0 + wm * T::WTM, n0 + wn * T::WTN, relu, g,
        t, vec4, addend,
        args.split_k == 1 && (args.epilogue & HEXIR_EPILOGUE_STREAM) != 0);
    if (args.split_k == 1 && (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE))
      __threadfence_system();
  }
  // Nothing may still be writing this CTA's shared memory when it exits.
  // Once every warp is past its loop no stage is armed again; wait for the
  // phase of each stage's last arm (at once after a normal run, where every
  // arm was waited for).
  __syncthreads();
  if (issuer) {
    const int32_t issued = (int32_t)*(volatile uint32_t *)armed;
#pragma unroll
    for (int s = 0; s < STAGES; ++s)
      if (issued > s) {
        const uint32_t uses = (uint32_t)(issued - s + STAGES - 1) / STAGES;
        mbar_wait_bounded(&full[s], (uses - 1) & 1u, args.timeout_ns);
      }
  }
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
  // Stage releases and arms, as in linear_tma_body.
  uint32_t *released = reinterpret_cast<uint32_t *>(full + STAGES);
  uint32_t *armed = released + STAGES;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool issuer = threadIdx.x == 0;
  const SkSteps steps(args);
  const int32_t nk = (int32_t)steps.n_steps;
  // The fix-up may start launching: the whole grid is resident (one CTA
  // per SM), so its CTAs only take SMs this grid has left.
  griddep_launch_dependents();

  if (issuer) {
    prefetch_tensormap(map_a);
    prefetch_tensormap(map_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      released[s] = 0u;
    }
    *armed = (uint32_t)min(nk, (int32_t)STAGES);
    fence_mbar_init();
  }
  __syncthreads();

  // Arm stage i % STAGES for the step at cursor `at` and issue its boxes.
  // Thread 0 issues the first STAGES steps; after that the warp that
  // releases a stage last refills it with the step STAGES ahead, which
  // every warp tracks with its own cursor (`ahead`), with the row / column
  // of that cursor's tile cached.
  uint32_t at_tile = ~0u, atm = 0, atn = 0;
  auto issue = [&](int32_t i, const SkSteps::Cursor &at) {
    const int s = i % STAGES;
    if (at.tile != at_tile) {
      at_tile = at.tile;
      tile_of(at_tile, args.tiles_m, args.tiles_n, args.group_m, atm, atn);
    }
    mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
    const int32_t k0 = (int32_t)(at.kt * BK);
    double *as = sa + s * T::A_STAGE;
    double *bs = sb + s * T::B_STAGE;
#pragma unroll
    for (int j = 0; j < BK / 8; ++j)
      tma_load_2d(as + j * T::A_SLAB, map_a, k0 + j * 8, (int32_t)(atm * BM),
                  &full[s]);
#pragma unroll
    for (int j = 0; j < BN / 16; ++j)
      tma_load_2d(bs + j * T::B_SLAB, map_b, (int32_t)(atn * BN + j * 16), k0,
                  &full[s]);
  };
  SkSteps::Cursor ahead = steps.begin();
  for (int32_t j = 0; j < nk && j < STAGES; ++j) {
    if (issuer)
      issue(j, ahead);
    steps.next(ahead);
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
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&full[s], use & 1u, args.timeout_ns))) {
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
      // Release stage s; the last of its 8 releases refills it with the
      // step STAGES ahead (see linear_tma_body).
      if (lane == 0) {
        const uint32_t before = atom_add_acq_rel_cta(&released[s], 1u);
        if (before % HEXIR_LINEAR_CONSUMER_WARPS ==
                HEXIR_LINEAR_CONSUMER_WARPS - 1 &&
            i + STAGES < nk) {
          issue(i + STAGES, ahead);
          atomicAdd(armed, 1u);
        }
      }
      steps.next(ahead);
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

  if (ok && (args.epilogue & HEXIR_EPILOGUE_SYSTEM_FENCE))
    __threadfence_system();
  // Nothing may still be writing this CTA's shared memory when it exits
  // (see linear_tma_body).
  __syncthreads();
  if (issuer) {
    const int32_t issued = (int32_t)*(volatile uint32_t *)armed;
#pragma unroll
    for (int s = 0; s < STAGES; ++s)
      if (issued > s) {
        const uint32_t uses = (uint32_t)(issued - s + STAGES - 1) / STAGES;
        mbar_wait_bounded(&full[s], (uses - 1) & 1u, args.timeout_ns);
      }
  }
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

// Completes the stream-K tiles whose k units were split over CTAs: the
// partial tiles are summed in CTA order (the order of k), then the epilogue
// (addend, relu) applies.  Tiles owned by one CTA were stored by it and are
// skipped.  Grid (tiles, HEXIR_SK_FIXUP_PARTS): each CTA takes every
// PARTS-th group of four consecutive columns of its tile, so a thread has
// one 256-bit load per partial in flight instead of walking the tile
// element by element (one CTA per tile left each thread 64 dependent
// trips to memory, longer than the whole stream-K loop at 1024^3).
extern "C" __global__ void __launch_bounds__(256)
    hexir_linear_f64_sk_fixup(const hexir_linear_args_t args) {
  constexpr uint32_t BM = HEXIR_LINEAR_BM, BN = HEXIR_LINEAR_BN;
  griddep_wait();  // the stream-K grid's partial tiles
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
  const bool vec4 = (args.epilogue & HEXIR_EPILOGUE_VEC4) != 0;
  const uint32_t stride = gridDim.y * blockDim.x * 4u;
  for (uint32_t e = (blockIdx.y * blockDim.x + threadIdx.x) * 4u; e < BM * BN;
       e += stride) {
    const uint32_t r = e / BN, col = e % BN;
    const uint32_t row = tm * BM + r, gcol = tn * BN + col;
    if (row >= args.m || gcol >= args.n)
      continue;
    double s[4] = {0.0, 0.0, 0.0, 0.0};
    for (uint32_t c = c0; c <= c1; ++c) {
      // The CTA's run starts in this tile: its first-tile slot.
      const uint32_t first = args.sk_dp_tiles + (c * U) / k_tiles;
      const uint32_t slot = 2 * c + (tile == first ? 0u : 1u);
      // Slots are 32-byte aligned (the workspace base is) and e % 4 == 0.
      double v[4];
      ldg256(args.sk_partials + (size_t)slot * BM * BN + e, v);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        s[q] = __dadd_rn(s[q], v[q]);
    }
    const size_t idx = (size_t)row * args.n + gcol;
    if (vec4) {
      // Rows of c and the addend start 32-byte aligned and n % 4 == 0, so
      // the four columns are in range together.
      if (add) {
        double a4[4];
        ldg256(args.addend + idx, a4);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          s[q] = __dadd_rn(s[q], a4[q]);
      }
      if (relu) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          s[q] = relu_ref(s[q]);
      }
      stg256(args.c + idx, s[0], s[1], s[2], s[3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (gcol + q < args.n) {
          double x = s[q];
          if (add)
            x = __dadd_rn(x, args.addend[idx + q]);
          args.c[idx + q] = relu ? relu_ref(x) : x;
        }
      }
    }
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
