// linear_tiles.cuh -- the DMMA building blocks shared by the f64 linear
// kernels (linear_f64.cu: the TMA-fed kernels; linear_guarded_f64.cu: the
// bounds-checked kernel and the split-K reduction): the tile raster, one k8
// step of a warp tile, and the warp tile's loads and stores.
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
#pragma once

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
