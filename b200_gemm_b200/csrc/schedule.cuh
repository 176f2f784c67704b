// Persistent tile schedule: the output is cut into 256x256 tiles (one per
// CTA pair) and the tiles are ordered along a Hilbert curve so that the tiles
// in flight at the same moment share rows of A and columns of B in L2.
//
// Reference: include/hilbert.hpp:11-84 (`hilbert_d2xy`, `createHilbert`),
// called from b200_kernels/matmul_1.cuh:401.  The curve walk (index ->
// cell) is the published Hilbert d2xy construction, so it has to produce the
// same cells as the reference's; the assignment to clusters differs: here the
// ordered list is dealt out round-robin over every cluster of the grid (entry
// j runs on cluster j mod G), which keeps all clusters within one tile of each
// other instead of filling 64 clusters first (hilbert.hpp:47-77).
#pragma once

#include <cstdint>

namespace b200gemm {

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

// One CTA of 1024 threads walks the curve over the padded square and writes
// the in-range cells, in curve order, to out[0 .. tiles_m*tiles_n).
__global__ void __launch_bounds__(1024) build_hilbert_schedule_kernel(uint32_t tiles_m, uint32_t tiles_n,
                                                                      uint32_t* __restrict__ out) {
  __shared__ uint32_t warp_count[32];
  __shared__ uint32_t warp_base[32];
  __shared__ uint32_t chunk_total;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
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

}  // namespace b200gemm
