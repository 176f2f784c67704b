// Persistent tile schedule.  The output is cut into 256 x 256 tiles (one per
// CTA pair); a schedule is the list of all tiles in the order they start.
// Entry j runs on cluster j mod G (G = clusters in the grid), so at any
// moment the G tiles in flight are G consecutive entries: the order decides
// which rows of A and columns of B they share in L2.
//
// Two orders:
//   * Hilbert curve over the tile grid (reference include/hilbert.hpp:11-84,
//     `hilbert_d2xy` / `createHilbert`, used at matmul_1.cuh:401).  The
//     index -> cell walk is the published Hilbert d2xy construction, so it
//     visits the same cells in the same order as the reference's.  The
//     reference then deals tiles to its first 64 clusters and moves a tail to
//     the other 10 (hilbert.hpp:47-77); here every cluster gets every G-th
//     entry, which keeps all clusters within one tile of each other.
//   * Row bands: bands of `band` tile-rows; inside a band the columns are
//     swept one at a time (all rows of the band for a column, then the next
//     column), alternating direction from band to band.  The A rows of a band
//     stay in L2 while the whole of B streams past once per band.
#pragma once

#include <cstdint>

namespace b200gemm {

enum : int { kOrderHilbert = 0, kOrderBands = 1 };

// Cell (x, y) visited at step d of the Hilbert curve over a side x side grid
// (side a power of two).
__host__ __device__ inline void hilbert_cell(uint32_t side, uint32_t d, uint32_t& x, uint32_t& y) {
  uint32_t px = 0, py = 0;
  for (uint32_t s = 1; s < side; s <<= 1) {
    const uint32_t rx = (d >> 1) & 1u;
    const uint32_t ry = (d ^ rx) & 1u;
    if (ry == 0) {  // rotate the sub-square
      if (rx == 1) {
        px = s - 1 - px;
        py = s - 1 - py;
      }
      const uint32_t t = px;
      px = py;
      py = t;
    }
    px += s * rx;
    py += s * ry;
    d >>= 2;
  }
  x = px;
  y = py;
}

__host__ __device__ inline uint32_t hilbert_side(uint32_t tiles_m, uint32_t tiles_n) {
  uint32_t m = tiles_m > tiles_n ? tiles_m : tiles_n;
  uint32_t side = 1;
  while (side < m) side <<= 1;
  return side;
}

// Tile ids are packed as (tile_m << 16) | tile_n.
__host__ __device__ inline uint32_t pack_tile(uint32_t tm, uint32_t tn) { return (tm << 16) | tn; }

// Entry i of the row-band order (closed form).
__host__ __device__ inline uint32_t band_tile(uint32_t i, uint32_t tiles_m, uint32_t tiles_n,
                                              uint32_t band) {
  const uint32_t per_band = band * tiles_n;
  const uint32_t b = i / per_band;
  const uint32_t o = i - b * per_band;
  const uint32_t row0 = b * band;
  const uint32_t rows = (tiles_m - row0 < band) ? tiles_m - row0 : band;
  uint32_t col = o / rows;
  const uint32_t r = o - col * rows;
  if (b & 1u) col = tiles_n - 1 - col;
  return pack_tile(row0 + r, col);
}

// Writes the schedule for a tiles_m x tiles_n grid to out[0 .. tiles_m*tiles_n).
// One CTA of 1024 threads.  For the Hilbert order it walks the curve over the
// padded square and compacts the in-range cells with a block-wide scan.
__global__ void __launch_bounds__(1024) build_schedule_kernel(uint32_t tiles_m, uint32_t tiles_n,
                                                              int order, uint32_t band,
                                                              uint32_t* __restrict__ out) {
  const uint32_t tid = threadIdx.x;
  const uint64_t total = static_cast<uint64_t>(tiles_m) * tiles_n;
  if (order == kOrderBands) {
    for (uint64_t i = tid; i < total; i += 1024)
      out[i] = band_tile(static_cast<uint32_t>(i), tiles_m, tiles_n, band);
    return;
  }
  __shared__ uint32_t warp_count[32];
  __shared__ uint32_t warp_base[32];
  __shared__ uint32_t chunk_total;
  const uint32_t lane = tid & 31u, warp = tid >> 5;
  const uint32_t side = hilbert_side(tiles_m, tiles_n);
  const uint64_t cells = static_cast<uint64_t>(side) * side;
  uint32_t written = 0;
  for (uint64_t chunk = 0; chunk < cells; chunk += 1024) {
    const uint64_t d = chunk + tid;
    uint32_t x = 0, y = 0;
    bool keep = false;
    if (d < cells) {
      hilbert_cell(side, static_cast<uint32_t>(d), x, y);
      keep = (x < tiles_m) && (y < tiles_n);
    }
    const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
    const uint32_t rank_in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_count[warp] = __popc(ballot);
    __syncthreads();
    if (warp == 0) {
      const uint32_t c = warp_count[lane];
      uint32_t incl = c;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += v;
      }
      warp_base[lane] = incl - c;
      if (lane == 31) chunk_total = incl;
    }
    __syncthreads();
    if (keep) out[written + warp_base[warp] + rank_in_warp] = pack_tile(x, y);
    written += chunk_total;
    __syncthreads();
  }
}

// Host mirror of build_schedule_kernel (same output).
inline void build_schedule_host(uint32_t tiles_m, uint32_t tiles_n, int order, uint32_t band,
                                uint32_t* out) {
  const uint64_t total = static_cast<uint64_t>(tiles_m) * tiles_n;
  if (order == kOrderBands) {
    for (uint64_t i = 0; i < total; ++i) out[i] = band_tile(static_cast<uint32_t>(i), tiles_m, tiles_n, band);
    return;
  }
  const uint32_t side = hilbert_side(tiles_m, tiles_n);
  const uint64_t cells = static_cast<uint64_t>(side) * side;
  uint64_t w = 0;
  for (uint64_t d = 0; d < cells; ++d) {
    uint32_t x, y;
    hilbert_cell(side, static_cast<uint32_t>(d), x, y);
    if (x < tiles_m && y < tiles_n) out[w++] = pack_tile(x, y);
  }
}

}  // namespace b200gemm
