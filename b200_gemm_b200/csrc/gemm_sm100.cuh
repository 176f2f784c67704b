// Persistent, warp-specialised bf16 GEMM for sm_100a:
//   C[M x N] (bf16, row-major, leading dim ldc) = A[M x K] . B[N x K]^T
// with A and B row-major ("K-major") bf16 and fp32 accumulation in TMEM.
//
// Reference path: b200_kernels/matmul_1.cuh:329-381 (`matmulKernel1`) and
// its helpers (tma_warp :158-196, mma_warp :209-261, epilogue :270-319).
// Same contract and the same per-pair MMA tile (256 x 256, K step 16,
// cta_group::2); the pipeline around it is rebuilt:
//   * the smem ring is initialised once and runs across tiles (the
//     reference re-initialises every barrier and cluster-syncs per tile,
//     matmul_1.cuh:373-374);
//   * 256-column tiles: two TMEM accumulators (2 x 256 fp32 columns) let the
//     MMA warp start tile i+1 while four dedicated epilogue warps drain tile
//     i; 256 x 512 tiles (two MMAs per K step sharing the A stage) fill TMEM
//     with one accumulator, which 8 epilogue warps read out completely
//     (into staging buffers and registers) before any store, so the next
//     tile's MMAs wait only for the TMEM reads;
//   * the epilogue reads 32 columns per tcgen05.ld, converts to bf16 (RNE),
//     writes 64B-swizzled staging buffers (bank-conflict free) and streams
//     them out with per-warp TMA stores;
//   * ragged M, N and K (K % 8 == 0) are handled by TMA bounds (zero fill on
//     loads, clipping on stores) instead of requiring multiples of 256/64;
//     the one chunk that ends inside a 16-byte group when N % 8 != 0 is
//     stored element by element;
//   * every wait is bounded (see ptx_sm100.cuh).
//
// Warp roles (64 + 32 x EW threads per CTA, one CTA per SM, clusters of 2):
//   warp 0      TMA producer (one lane), both CTAs
//   warp 1      MMA issuer (one lane), leader CTA only; TMEM allocator
//   warps 2..   EW epilogue warps; warp w reads TMEM lanes 32*(w%4) .. +31
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "ptx_sm100.cuh"

// L2 eviction priority of the operand loads (0 normal, 1 evict_last,
// 2 evict_first); build-time tuning knobs.  Both operands evict_last: the
// C tiles the epilogue writes then leave L2 before A or B lines do (measured
// 0.3-0.8% faster than A normal across 8192^3, the MLP shapes and 16384 x
// 2048 x 16384, with the same DRAM bytes).
#ifndef B200GEMM_L2_POLICY_A
#define B200GEMM_L2_POLICY_A 1
#endif
#ifndef B200GEMM_L2_POLICY_B
#define B200GEMM_L2_POLICY_B 1
#endif
// Staging buffers per epilogue warp of the plain 256 x 512 instances.
#ifndef B200GEMM_CBUFS_N512
#define B200GEMM_CBUFS_N512 4
#endif
// The same for the fused-epilogue shared-A instances.
#ifndef B200GEMM_CBUFS_E512
#define B200GEMM_CBUFS_E512 2
#endif


namespace b200gemm {

constexpr int kTileM = 256;       // rows of C per CTA pair (128 per CTA)
constexpr int kBlockN = 256;      // columns per tcgen05.mma (N of one instruction)
constexpr int kBlockK = 64;       // K per pipeline stage: one 128-byte swizzle row of bf16
constexpr int kMmaK = 16;         // K per tcgen05.mma (kind::f16)
constexpr int kTmemCols = 512;    // the whole TMEM of the SM
constexpr int kStageBytesA = 128 * kBlockK * 2;       // A rows of one CTA, one stage
constexpr int kCBoxCols = 32;     // one 64-byte row of bf16 (64-byte swizzle)
constexpr int kCBoxRows = 32;     // one warp's TMEM lane quarter
constexpr int kCStageBytes = kCBoxCols * kCBoxRows * 2;  // 2 KB staging buffer

// Watchdog sites (reported in status word 1).
enum : unsigned int {
  kSiteProducer = 1,
  kSiteMmaTmemEmpty = 2,
  kSiteMmaFull = 3,
  kSiteEpilogue = 4,
  kSiteDrain = 5,
  kSiteSelftest = 9,
};

struct GemmParams {
  int M, N, K;
  int num_kb;                 // ceil(K / kBlockK)
  int num_tiles;              // ceil(M / 256) * ceil(N / tile width)
  const uint32_t* tiles;      // schedule: num_tiles packed (tm << 16 | tn) in start order
  // Single-wave grids (every tile starts at once, so the order is moot):
  // whole tile u is (u / direct_tiles_n, u % direct_tiles_n), computed
  // instead of loaded from `tiles`; 0 = use the table.
  int direct_tiles_n;
  unsigned int* status;       // 4 status words (code, site, cta, tile); may be null
  unsigned long long timeout_ns;
  uint16_t* C;                // C base (bf16 bits), for the ragged-N edge chunk
  long long ldc;              // C row pitch in elements
  // Fused all-gather: every staged C chunk is also written to these peer
  // copies of C (IPC-mapped device memory on other GPUs, same pitch ldc,
  // already offset to this rank's first column).  npeers = 0 disables it.
  static constexpr int kMaxPeers = 7;
  int npeers;
  uint8_t* peer_c[kMaxPeers];
  // Fused all-gather through NVLink multicast: the multicast address of
  // this rank's first column of C (same pitch ldc), or null.  Every staged
  // chunk is written once with multimem.st; NVSwitch delivers it to every
  // GPU of the multicast object, this one included, so the chunk is not
  // also TMA-stored locally.
  uint8_t* mc_c;
  // Split of the last, partial wave: work units [0, tail_start) are whole
  // tiles (tiles[u]); unit tail_start + r * tail_split + s is K slice s (of
  // tail_kb K blocks) of tile tiles[tail_start + r].  A K slice writes its
  // fp32 partial to workspace and takes a ticket from tail_counters; the last
  // of a tile's slices adds the others to its own accumulator and stores C.
  int num_units;        // tail_start + tail_tiles * tail_split (or * 2 with tail_half)
  int tail_start;
  int tail_split;       // 1 = no split
  int tail_kb;
  // Shared-A tiles (NB = 2) only: with tail_half, unit tail_start + 2 r + h is the
  // h-th 256-column half of tile tiles[tail_start + r] over the whole of K,
  // so a last wave of up to half the clusters' tiles runs in about half a
  // tile's time on twice the clusters.
  int tail_half;
  float* workspace;     // [tail unit][CTA of the pair][128 rows x tile width] fp32
  unsigned int* tail_counters;  // [tail tile][CTA of the pair], zero between launches
  // Fused epilogue (instances with Cfg::kEpi only), per element in fp32:
  //   D = act(alpha * acc + bias[col]) + beta * residual[row][col]
  // then rounded to bf16 (RNE), stored as fp32, or scaled by out_scale and
  // rounded to fp8 e4m3 (RNE, saturating), per out_type.
  uint32_t epi_flags;          // kEpiBias | kEpiResidual
  int act;                     // kAct*
  int out_type;                // kOutBf16, kOutF32 (ldc in fp32), kOutE4m3 (ldc in bytes)
  float alpha, beta, out_scale;
  const uint16_t* bias;        // bf16[N]
  const uint16_t* residual;    // bf16, row pitch ldr elements
  long long ldr;
  int pdl;                     // kPdlOff or kPdlOn (launch overlap with the previous kernel)
};

constexpr uint32_t kEpiBias = 1u;
constexpr uint32_t kEpiResidual = 2u;
constexpr int kActNone = 0, kActRelu = 1, kActGelu = 2, kActGeluTanh = 3, kActSilu = 4;
constexpr int kOutBf16 = 0, kOutF32 = 1, kOutE4m3 = 2;
// Launch overlap with the previous kernel on the stream (programmatic
// dependent launch): off; on (the prologue overlaps, every global access
// waits for the previous kernel); on with B, the weights, streamed before
// that wait (small-M kernels only; the previous kernel must not write B).
constexpr int kPdlOff = 0, kPdlOn = 1, kPdlWeightsEarly = 2;

// One work unit of a CTA pair: a tile and a K range; slot >= 0 marks a K
// slice of a split tile (its index among the tail units), slot -2 - h the
// h-th 256-column half of a 256 x 512 tile, slot -1 a whole tile.
struct WorkUnit {
  uint32_t tile;
  int kb_begin, kb_end;
  int slot;
};

// Which 256-column half of a 256 x 512 tile a unit covers (-1: all of it).
__device__ __forceinline__ int unit_half(const WorkUnit& w) { return w.slot <= -2 ? -2 - w.slot : -1; }

template <bool HALF>
__device__ __forceinline__ WorkUnit unit_at(const GemmParams& p, uint32_t u) {
  WorkUnit w;
  if (u < static_cast<uint32_t>(p.tail_start)) {
    w.tile = p.direct_tiles_n > 0
                 ? ((u / static_cast<uint32_t>(p.direct_tiles_n)) << 16) | (u % static_cast<uint32_t>(p.direct_tiles_n))
                 : __ldg(p.tiles + u);
    w.kb_begin = 0;
    w.kb_end = p.num_kb;
    w.slot = -1;
  } else if (HALF) {
    const int v = static_cast<int>(u) - p.tail_start;
    w.tile = __ldg(p.tiles + p.tail_start + (v >> 1));
    w.kb_begin = 0;
    w.kb_end = p.num_kb;
    w.slot = -2 - (v & 1);
  } else {
    const int v = static_cast<int>(u) - p.tail_start;
    const int r = v / p.tail_split, sl = v - r * p.tail_split;
    w.tile = __ldg(p.tiles + p.tail_start + r);
    w.kb_begin = sl * p.tail_kb;
    w.kb_end = min(p.num_kb, w.kb_begin + p.tail_kb);
    w.slot = v;
  }
  return w;
}

// Compile-time shape of one kernel instance.
//   NB = 1: a pair computes 256 x 256 tiles; TMEM holds two accumulators, so
//           the MMA of tile i+1 overlaps the epilogue of tile i.
//   NB = 2: a pair computes 256 x 2MN tiles (MN = 256 or 224) as two N = MN
//           MMAs per K step that share the A stage: 25% fewer operand bytes
//           into each SM per flop than 256 x 256 tiles; the single 2MN-column
//           accumulator is drained by EW warps.  256 x 448 tiles divide
//           N = 1792 (the 8-way shard of a 14336-wide MLP projection).
//   MN (NB = 1 only): columns of one MMA and of the tile, a multiple of 32
//           up to 256 (e.g. 224 = 1792 / 8 for an N-sharded MLP projection),
//           so the tile width can divide N and fill the last wave.
//   EPI:    fused epilogue (bias, activation, residual, fp32 output) compiled
//           in; the plain instances carry none of its code.
//   EW:     epilogue warps (a multiple of 4; warp w reads TMEM lanes
//           32 (w % 4) ..); each drains kTileN * 4 / EW columns of its lanes.
//           More warps drain a single (non double-buffered) accumulator
//           sooner: every warp's chunks run as one serial chain of TMEM load,
//           staging and TMA store.
template <int STAGES, int NB, int MN = 256, bool EPI = false, int EW = 4 * NB, bool HALF = false>
struct GemmCfg {
  static_assert(NB == 1 || NB == 2, "one or two MMA column blocks per tile");
  static_assert(MN % 32 == 0 && MN >= 64 && MN <= 256 && (NB == 1 || MN == 256 || MN == 224), "MMA width");
  static constexpr int kStages = STAGES;
  static constexpr int kNB = NB;
  static constexpr bool kEpi = EPI;
  // Instances that run a short last wave as 256-column halves (tail_half);
  // a separate instance, so the others carry none of its code.
  static constexpr bool kHalfTail = HALF;
  static_assert(!HALF || (NB == 2 && !EPI), "half-width units are 256 x 512 plain tiles");
  static constexpr int kMmaN = MN;                       // columns per tcgen05.mma
  static constexpr int kBRows = MN / 2;                  // B rows per CTA per column block
  static constexpr int kBlockBytesB = kBRows * kBlockK * 2;
  static constexpr int kChunks = MN / kCBoxCols;         // 32-column chunks per MMA column block
  static constexpr int kTileN = MN * NB;
  static constexpr int kAccBufs = NB == 1 ? 2 : 1;
  static constexpr int kAccStride = 256;                 // TMEM column of accumulator 1
  // kind::f16: D f32, A = B = bf16, K-major, M = 256 (pair), N = MN.
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                     (static_cast<uint32_t>(MN >> 3) << 17) | ((kTileM >> 4) << 24);
  static constexpr int kEpiWarps = EW;
  static constexpr int kColsPerWarp = MN * NB * 4 / EW;       // tile columns one epilogue warp drains
  static constexpr int kWarpChunks = kColsPerWarp / kCBoxCols;
  static_assert(EW % 4 == 0 && kColsPerWarp % kCBoxCols == 0 && kWarpChunks >= 1, "epilogue warps");
  // K-split tail units (fp32 partials + reduction) are compiled into the
  // plain 256-column-MMA-block instances with one column block (in the
  // 512-wide instance the split only tied the narrower tiles and cost
  // registers); the host splits no other.
  static constexpr bool kTailSplit = !EPI && NB == 1 && EW <= 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  // Staging buffers per epilogue warp: a chunk's buffer is free once the
  // TMA store issued kCBufs chunks earlier has read it (about a microsecond),
  // so more buffers let a warp drain its accumulator faster.
  static constexpr int kCBufs = NB == 2 ? (EPI ? B200GEMM_CBUFS_E512 : B200GEMM_CBUFS_N512) : 2;
  // Plain instances with one accumulator: every epilogue warp reads all its
  // chunks from TMEM before any TMA store, the first kCBufs into its staging
  // buffers and the rest into registers, so the accumulator is released
  // after the TMEM reads alone (epilogue of gemm_bf16_nt_sm100).  Loads go
  // in pairs.
  static constexpr int kHeldChunks = kWarpChunks - kCBufs;
  static constexpr bool kStagedDrain = !EPI && NB == 2 && kHeldChunks > 0;
  static constexpr int kStageBytesB = kBlockBytesB * NB;
  static constexpr uint32_t kTxBytes = 2 * (kStageBytesA + kStageBytesB);  // both CTAs
  // shared memory layout (offsets from a 1024-byte aligned base)
  static constexpr int kA = 0;
  static constexpr int kB = kA + STAGES * kStageBytesA;
  static constexpr int kC = kB + STAGES * kStageBytesB;
  static constexpr int kFull = kC + kEpiWarps * kCBufs * kCStageBytes;
  static constexpr int kEmpty = kFull + 8 * STAGES;
  // Half units (kHalfTail) move one B block per K block, so once a CTA's
  // whole tiles are done its ring is re-cut into kHalfStages stages of
  // kHalfStageBytes (A, then the B block) over the same bytes, with their own
  // barriers: more bytes in flight than the whole-tile stages would carry.
  static constexpr int kHalfStageBytes = kStageBytesA + kBlockBytesB;
  static constexpr int kHalfStages = HALF ? STAGES * (kStageBytesA + kStageBytesB) / kHalfStageBytes : 0;
  static constexpr int kFull2 = kEmpty + 8 * STAGES;
  static constexpr int kEmpty2 = kFull2 + 8 * kHalfStages;
  static constexpr int kTFull = kEmpty2 + 8 * kHalfStages;
  static constexpr int kTEmpty = kTFull + 8 * kAccBufs;
  static constexpr int kDrain = kTEmpty + 8 * kAccBufs;
  static constexpr int kTmemSlot = kDrain + 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kTicket = kAbort + 4;     // "this CTA is the last K slice" flag
  static constexpr int kEnd = kTicket + 4;
  static constexpr int kSmemBytes = kEnd + 1024;  // slack to align the base to 1024 B
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
};

// Shared-memory matrix descriptor fields above the start address for a
// K-major operand in the 128-byte swizzle layout written by TMA: 8-row groups
// 1024 B apart (SBO), descriptor version 1, swizzle mode 2 (128 B).
constexpr uint64_t kSmemDescHi = (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 16)  // LBO unused
                                 | (uint64_t(1) << 46) | (uint64_t(2) << 61);

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return kSmemDescHi | uint64_t((addr & 0x3FFFFu) >> 4);
}

// Write one 32-row x 64-byte chunk of C: lane = row, w[] = the row's 16
// 32-bit words, i.e. 32 bf16 columns (packed pairs, ESIZE 2) or 16 fp32
// columns (ESIZE 4) starting at `col`.  Full chunks go through a 64-byte-
// swizzled staging buffer (16-byte group j of row r sits at group
// j ^ ((r >> 1) & 3), so the eight rows of each shared-memory wavefront hit
// distinct banks) and a TMA store.  TMA clips the innermost dimension in
// 16-byte units, so the chunk that ends inside a 16-byte group (N not a
// multiple of 16 / ESIZE) is written with per-element predicated stores.
// The 16 words of one lane (one row of a 32 x 64-byte chunk) into staging
// buffer `buf`, 64-byte swizzled (see store_c_chunk).
__device__ __forceinline__ void stage_chunk_row(uint32_t buf, uint32_t lane, const uint32_t (&w)[16]) {
  const uint32_t rowaddr = buf + lane * 64u;
  const uint32_t sw = (lane >> 1) & 3u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    ptx::st_shared_v4(rowaddr + ((static_cast<uint32_t>(j) ^ sw) << 4), w[4 * j], w[4 * j + 1], w[4 * j + 2],
                      w[4 * j + 3]);
  }
}

// The same from 32 fp32 accumulators, rounded to bf16 (RNE) pairwise as
// they are written, so no packed copy of the chunk is held.
__device__ __forceinline__ void stage_chunk_row_f32(uint32_t buf, uint32_t lane, const uint32_t (&v)[32]) {
  const uint32_t rowaddr = buf + lane * 64u;
  const uint32_t sw = (lane >> 1) & 3u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    ptx::st_shared_v4(rowaddr + ((static_cast<uint32_t>(j) ^ sw) << 4), ptx::pack_bf16x2(v[8 * j], v[8 * j + 1]),
                      ptx::pack_bf16x2(v[8 * j + 2], v[8 * j + 3]), ptx::pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                      ptx::pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
  }
}

// Fused all-gather: copy a staged chunk (rows row.., columns col.. of this
// rank's block) to every peer's C over NVLink: 32 rows x 64 B = 128
// segments of 16 B; four consecutive lanes write one row's 64 B.  The
// chunk must be staged and the warp synchronised.
template <int ESIZE>
__device__ __forceinline__ void copy_chunk_to_peers(uint32_t buf, int col, int row, uint32_t lane,
                                                    const GemmParams& p) {
  constexpr int kGroup = 16 / ESIZE;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const uint32_t seg = static_cast<uint32_t>(it) * 32u + lane;
    const uint32_t r = seg >> 2, q = seg & 3u;
    uint32_t x0, x1, x2, x3;
    ptx::ld_shared_v4(buf + r * 64u + ((q ^ ((r >> 1) & 3u)) << 4), x0, x1, x2, x3);
    const int grow = row + static_cast<int>(r), gcol = col + static_cast<int>(q) * kGroup;
    if (grow < p.M && gcol < p.N) {
      const long long off = (static_cast<long long>(grow) * p.ldc + gcol) * ESIZE;
      for (int i = 0; i < p.npeers; ++i) ptx::st_global_v4(p.peer_c[i] + off, x0, x1, x2, x3);
    }
  }
}

// Fused all-gather through NVLink multicast: write a staged chunk once to
// the multicast address, same segment order as copy_chunk_to_peers.
template <int ESIZE>
__device__ __forceinline__ void copy_chunk_to_multicast(uint32_t buf, int col, int row, uint32_t lane,
                                                        const GemmParams& p) {
  constexpr int kGroup = 16 / ESIZE;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const uint32_t seg = static_cast<uint32_t>(it) * 32u + lane;
    const uint32_t r = seg >> 2, q = seg & 3u;
    uint32_t x0, x1, x2, x3;
    ptx::ld_shared_v4(buf + r * 64u + ((q ^ ((r >> 1) & 3u)) << 4), x0, x1, x2, x3);
    const int grow = row + static_cast<int>(r), gcol = col + static_cast<int>(q) * kGroup;
    if (grow < p.M && gcol < p.N)
      ptx::multimem_st_v4(p.mc_c + (static_cast<long long>(grow) * p.ldc + gcol) * ESIZE, x0, x1, x2, x3);
  }
}

template <class Cfg, int ESIZE = 2>
__device__ __forceinline__ void store_c_chunk(const uint32_t (&w)[16], int col, int row,
                                              uint32_t lane, uint32_t cstage0, uint32_t& cbuf,
                                              const CUtensorMap& map_c, const GemmParams& p) {
  static_assert(ESIZE == 2 || ESIZE == 4, "bf16 or fp32 C");
  constexpr int kCols = 64 / ESIZE;        // columns per chunk
  constexpr int kGroup = 16 / ESIZE;       // columns per 16-byte group
  const bool store = (row < p.M) && (col < p.N);  // warp-uniform
  const bool ragged = ((p.N % kGroup) != 0) && (col + kCols > p.N);
  if (store && ragged) {
    const int r = row + static_cast<int>(lane);
    if (r < p.M) {
      const int ncols = p.N - col;
      if constexpr (ESIZE == 2) {
        uint16_t* dst = p.C + static_cast<long long>(r) * p.ldc + col;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (2 * i < ncols) dst[2 * i] = static_cast<uint16_t>(w[i] & 0xFFFFu);
          if (2 * i + 1 < ncols) dst[2 * i + 1] = static_cast<uint16_t>(w[i] >> 16);
        }
      } else {
        uint32_t* dst = reinterpret_cast<uint32_t*>(p.C) + static_cast<long long>(r) * p.ldc + col;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < ncols) dst[i] = w[i];
      }
    }
  } else if (store) {
    const uint32_t buf = cstage0 + cbuf * kCStageBytes;
    // The TMA store that last read this buffer (two chunks ago) must be done.
    if (lane == 0) ptx::bulk_wait_group_read<Cfg::kCBufs - 1>();
    __syncwarp();
    stage_chunk_row(buf, lane, w);
    if (p.mc_c != nullptr) {
      __syncwarp();
      copy_chunk_to_multicast<ESIZE>(buf, col, row, lane, p);
      __syncwarp();  // every lane has read the buffer before it is reused
    } else {
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        ptx::tma_store_2d(&map_c, buf, col, row);
        ptx::bulk_commit_group();
      }
      if (p.npeers > 0) copy_chunk_to_peers<ESIZE>(buf, col, row, lane, p);
    }
    if (++cbuf == Cfg::kCBufs) cbuf = 0;
  }
}

// bf16 bits -> fp32.
__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xFFFF0000u); }

// Eight bf16 values src[col .. col + 7] as four packed pairs; columns at or
// past N read as 0.  The vector path needs src 16-byte aligned at col
// (checked on the host for bias and residual rows; col is a multiple of 8).
__device__ __forceinline__ void load_bf16x8(const uint16_t* src, int col, int N, uint32_t (&w)[4]) {
  if (col + 8 <= N) {
    ptx::ld_global_nc_v4(src + col, w[0], w[1], w[2], w[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = (col + 2 * i < N) ? __ldg(src + col + 2 * i) : 0u;
      const uint32_t hi = (col + 2 * i + 1 < N) ? __ldg(src + col + 2 * i + 1) : 0u;
      w[i] = lo | (hi << 16);
    }
  }
}

// Epilogue operands of one epilogue warp for one tile, loaded before the
// warp waits for the tile's accumulator so their latency hides behind it:
// the bias of the warp's MMA column block (lane l holds columns 8l .. 8l+7,
// handed to the other lanes by shuffles) and the residual row of the first
// 32-column chunk (then each next chunk's while the current one is done).
__device__ __forceinline__ void epi_load_bias(const GemmParams& p, int col0, int ncols, uint32_t lane,
                                              uint32_t (&bias_w)[4]) {
  const int c = col0 + 8 * static_cast<int>(lane);
  if ((p.epi_flags & kEpiBias) && 8 * static_cast<int>(lane) < ncols && c < p.N) {
    load_bf16x8(p.bias, c, p.N, bias_w);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) bias_w[i] = 0u;
  }
}

__device__ __forceinline__ void epi_load_residual(const GemmParams& p, int r, int col, uint32_t (&q)[16]) {
  if ((p.epi_flags & kEpiResidual) && r < p.M && col < p.N) {
    const uint16_t* src = p.residual + static_cast<long long>(r) * p.ldr;
    if (col + 32 <= p.N && (reinterpret_cast<uintptr_t>(src + col) & 31u) == 0) {
      // two 32-byte loads: half the L1 wavefronts of four 16-byte ones
      uint32_t w0[8], w1[8];
      ptx::ld_global_nc_v8(src + col, w0);
      ptx::ld_global_nc_v8(src + col + 16, w1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[i] = w0[i];
        q[8 + i] = w1[i];
      }
      return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
      load_bf16x8(src, col + 8 * j, p.N, w);
#pragma unroll
      for (int i = 0; i < 4; ++i) q[4 * j + i] = w[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) q[i] = 0u;
  }
}

// Fused-epilogue arguments of the small-M kernels (the tiled kernel keeps
// the same fields in GemmParams).
struct EpiArgs {
  uint32_t flags;             // kEpiBias | kEpiResidual
  int act;                    // kAct*
  int out_type;               // kOutBf16, kOutF32, kOutE4m3
  float alpha, beta, out_scale;
  const uint16_t* bias;       // bf16[N]
  const uint16_t* residual;   // bf16, row pitch ldr elements
  long long ldr;
};

// Small-M kernels: the thread owns C column `col`; acc[t] is C[row0 + t][col]
// (t < 32).  Applies D = act(alpha * acc + bias[col]) + beta * R[row][col]
// in place.  R comes from the warp's residual tile in shared memory (loaded
// by TMA, zeros outside M and N): element t of this thread at
// rtile + 64 t.  The activation switch sits outside straight 32-element
// loops: a switch per element spreads the executed instructions over the
// whole inlined code and misses the instruction cache at every element.
__device__ __forceinline__ void smallm_epilogue(float (&acc)[32], int col, const EpiArgs& e, int N,
                                                uint32_t rtile) {
  const bool in_n = col < N;
  const float b = ((e.flags & kEpiBias) && in_n) ? __uint_as_float(static_cast<uint32_t>(__ldg(e.bias + col)) << 16)
                                                 : 0.0f;
  const bool res = (e.flags & kEpiResidual) != 0u;
#pragma unroll
  for (int t = 0; t < 32; ++t) acc[t] = fmaf(e.alpha, acc[t], b);
  const bool fast = e.out_type != kOutF32;
  switch (e.act) {
    case kActRelu:
#pragma unroll
      for (int t = 0; t < 32; ++t) acc[t] = fmaxf(acc[t], 0.0f);
      break;
    case kActGelu:
#pragma unroll
      for (int t = 0; t < 32; ++t) acc[t] = 0.5f * acc[t] * (1.0f + erff(acc[t] * 0.70710678118654752f));
      break;
    case kActGeluTanh:
      if (fast) {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float x = acc[t];
          acc[t] = 0.5f * x * (1.0f + ptx::tanh_approx(0.79788456080286536f * fmaf(0.044715f * x, x * x, x)));
        }
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float x = acc[t];
          acc[t] = 0.5f * x * (1.0f + tanhf(0.79788456080286536f * (x + 0.044715f * x * x * x)));
        }
      }
      break;
    case kActSilu:
      if (fast) {
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[t] = acc[t] * ptx::rcp_approx(1.0f + __expf(-acc[t]));
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[t] = acc[t] / (1.0f + expf(-acc[t]));
      }
      break;
    default:
      break;
  }
  if (res) {
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      uint16_t r;
      asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(rtile + static_cast<uint32_t>(t) * 64u) : "memory");
      acc[t] = fmaf(e.beta, __uint_as_float(static_cast<uint32_t>(r) << 16), acc[t]);
    }
  }
}

// Small-M kernels: one chunk of 32 rows of C for the warp's 32 columns into
// the transposing staging buffer [rows][32 columns] in the output type
// (bf16: 64-byte rows, fp32: 128, e4m3: 32); `lane` = the column.
__device__ __forceinline__ void smallm_stage(const float (&acc)[32], uint32_t cw, int c, uint32_t lane,
                                             int out_type, float out_scale) {
  // One branch per chunk, straight loops inside (see smallm_epilogue).
  const uint32_t row0 = static_cast<uint32_t>(c * 32);
  if (out_type == kOutF32) {
#pragma unroll
    for (int t = 0; t < 32; ++t)
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(cw + (row0 + t) * 128u + lane * 4u), "r"(__float_as_uint(acc[t]))
                   : "memory");
  } else if (out_type == kOutE4m3) {
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const uint32_t q = ptx::pack_e4m3x4(out_scale * acc[t], 0.0f, 0.0f, 0.0f) & 0xFFu;
      asm volatile("st.shared.u8 [%0], %1;" ::"r"(cw + (row0 + t) * 32u + lane), "r"(q) : "memory");
    }
  } else {
#pragma unroll
    for (int t = 0; t < 32; ++t)
      ptx::st_shared_u16(cw + (row0 + t) * 64u + lane * 2u, __bfloat16_as_ushort(__float2bfloat16_rn(acc[t])));
  }
}

// One lane's 32 e4m3 bytes (8 words, column col + 4i + b in byte b of
// word i) to row r of C, straight from registers: two 16-byte stores when
// the chunk is whole (rows start 16-byte aligned: ldc % 16 == 0), else one
// byte per column inside N.
__device__ __forceinline__ void store_e4m3_row(const uint32_t (&q)[8], int r, int col, const GemmParams& p) {
  if (r >= p.M || col >= p.N) return;
  uint8_t* dst = reinterpret_cast<uint8_t*>(p.C) + static_cast<long long>(r) * p.ldc + col;
  if (col + 32 <= p.N) {
    ptx::st_global_v4(dst, q[0], q[1], q[2], q[3]);
    ptx::st_global_v4(dst + 16, q[4], q[5], q[6], q[7]);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (col + k < p.N) dst[k] = static_cast<uint8_t>(q[k >> 2] >> (8 * (k & 3)));
  }
}

// The fused epilogue on one lane's 32 accumulators (chunk `c` of the warp's
// column block), in place, fp32 throughout:
//   D = act(alpha * acc + bias[col]) + beta * residual[r][col].
// GELU is 0.5 x (1 + erf(x / sqrt 2)) or its tanh form
// 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))) (Hendrycks & Gimpel);
// SiLU is x / (1 + e^-x).  For fp32 output the transcendentals are CUDA's
// erff / tanhf / expf; for bf16 and e4m3 output, whose spacing (2^-8 and
// 2^-4 relative) is far coarser than their error, tanh and the reciprocal are
// the hardware approximations (tanh.approx, rcp.approx) and e^x is __expf.
// erf is erff for all.
__device__ __forceinline__ void apply_epilogue(uint32_t (&v)[32], int c, const uint32_t (&bias_w)[4],
                                               const uint32_t (&res_w)[16], const GemmParams& p) {
  float d[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) d[k] = p.alpha * __uint_as_float(v[k]);
  if (p.epi_flags & kEpiBias) {
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      // columns 32c + 2q, +1 live in lane 4c + q / 4, word q % 4
      const uint32_t b = __shfl_sync(0xFFFFFFFFu, bias_w[q & 3], 4 * c + (q >> 2));
      d[2 * q] += bf16_lo(b);
      d[2 * q + 1] += bf16_hi(b);
    }
  }
  const bool fast = p.out_type != kOutF32;
  switch (p.act) {
    case kActRelu:
#pragma unroll
      for (int k = 0; k < 32; ++k) d[k] = fmaxf(d[k], 0.0f);
      break;
    case kActGelu:
#pragma unroll
      for (int k = 0; k < 32; ++k) d[k] = 0.5f * d[k] * (1.0f + erff(d[k] * 0.70710678118654752f));
      break;
    case kActGeluTanh:
      if (fast) {
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float x = d[k];
          const float u = 0.79788456080286536f * fmaf(0.044715f * x, x * x, x);
          d[k] = 0.5f * x * (1.0f + ptx::tanh_approx(u));
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float x = d[k];
          d[k] = 0.5f * x * (1.0f + tanhf(0.79788456080286536f * (x + 0.044715f * x * x * x)));
        }
      }
      break;
    case kActSilu:
      if (fast) {
#pragma unroll
        for (int k = 0; k < 32; ++k) d[k] = d[k] * ptx::rcp_approx(1.0f + __expf(-d[k]));
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) d[k] = d[k] / (1.0f + expf(-d[k]));
      }
      break;
    default:
      break;
  }
  if (p.epi_flags & kEpiResidual) {
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      d[2 * q] = fmaf(p.beta, bf16_lo(res_w[q]), d[2 * q]);
      d[2 * q + 1] = fmaf(p.beta, bf16_hi(res_w[q]), d[2 * q + 1]);
    }
  }
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = __float_as_uint(d[k]);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1) __cluster_dims__(2, 1, 1)
    gemm_bf16_nt_sm100(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_c, const GemmParams p) {
  constexpr int STAGES = Cfg::kStages;
  constexpr int NB = Cfg::kNB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = (rank == 0);
  const uint32_t cluster = ptx::cluster_id_x();
  const uint32_t nclusters = ptx::num_clusters_x();

  const uint32_t sA = base + Cfg::kA, sB = base + Cfg::kB, sC = base + Cfg::kC;
  const uint32_t full0 = base + Cfg::kFull, empty0 = base + Cfg::kEmpty;
  const uint32_t tfull0 = base + Cfg::kTFull, tempty0 = base + Cfg::kTEmpty;
  const uint32_t drain = base + Cfg::kDrain, tmem_slot = base + Cfg::kTmemSlot;

  ptx::Watchdog wd;
  wd.abort_flag = base + Cfg::kAbort;
  wd.peer_abort_flag = ptx::mapa(wd.abort_flag, rank ^ 1u);
  wd.status = p.status;
  wd.timeout_ns = p.timeout_ns;

  if (threadIdx.x == 0) {
    asm volatile("st.shared.u32 [%0], 0;" ::"r"(wd.abort_flag) : "memory");
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full0 + 8 * s, 1);   // leader's expect_tx arrival (+ bytes of both CTAs)
      ptx::mbar_init(empty0 + 8 * s, 1);  // one MMA commit
    }
    for (int s = 0; s < Cfg::kHalfStages; ++s) {
      ptx::mbar_init(base + Cfg::kFull2 + 8 * s, 1);
      ptx::mbar_init(base + Cfg::kEmpty2 + 8 * s, 1);
    }
    for (int a = 0; a < Cfg::kAccBufs; ++a) {
      ptx::mbar_init(tfull0 + 8 * a, 1);                     // one MMA commit
      ptx::mbar_init(tempty0 + 8 * a, 2 * Cfg::kEpiWarps);   // every epilogue warp of the pair
    }
    ptx::mbar_init(drain, 1);
    ptx::fence_mbar_init_cluster();
    ptx::prefetch_tensormap(&map_a);
    ptx::prefetch_tensormap(&map_b);
    ptx::prefetch_tensormap(&map_c);
  }
  if (warp == 1) {
    ptx::tmem_alloc_cg2(tmem_slot, kTmemCols);
    ptx::tmem_relinquish_cg2();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync_all();
  ptx::tc_fence_after();
  uint32_t tmem_base;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem_base) : "r"(tmem_slot) : "memory");
  // Launched to overlap the previous kernel (kPdlOn), the setup above ran
  // during its tail; the tile table, A, B, C and the epilogue operands may
  // all be its output, so nothing global is touched before it completes.
  ptx::griddep_wait();

  const uint32_t num_units = static_cast<uint32_t>(p.num_units);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t policy_a = ptx::l2_policy(B200GEMM_L2_POLICY_A);
      const uint64_t policy_b = ptx::l2_policy(B200GEMM_L2_POLICY_B);
      const uint32_t full_leader0 = ptx::mapa(full0, 0);
      uint32_t stage = 0, phase = 0;
      [[maybe_unused]] uint32_t hstage = 0, hphase = 0;
      [[maybe_unused]] bool half_ring = false;
      bool ok = true;
      WorkUnit nxt = (cluster < num_units) ? unit_at<Cfg::kHalfTail>(p, cluster) : WorkUnit{0, 0, 0, -1};
      for (uint32_t t = cluster; t < num_units && ok; t += nclusters) {
        const WorkUnit cur = nxt;
        if (t + nclusters < num_units) nxt = unit_at<Cfg::kHalfTail>(p, t + nclusters);
        const uint32_t tile = cur.tile;
        const int row_a = static_cast<int>(tile >> 16) * kTileM + static_cast<int>(rank) * 128;
        const int row_b =
            static_cast<int>(tile & 0xFFFFu) * Cfg::kTileN + static_cast<int>(rank) * Cfg::kBRows;
        if constexpr (Cfg::kHalfTail) {
          if (cur.slot <= -2) {
            // Half units come after this CTA's whole tiles.  Before the ring
            // is re-cut, every whole-tile stage must have been consumed.
            if (!half_ring) {
              for (int s = 0; s < STAGES && ok; ++s) {
                if (!ptx::mbar_wait(empty0 + 8 * stage, phase ^ 1u, wd, kSiteProducer, t)) ok = false;
                if (++stage == STAGES) {
                  stage = 0;
                  phase ^= 1u;
                }
              }
              half_ring = true;
              if (!ok) break;
            }
            const uint32_t full2 = base + Cfg::kFull2, empty2 = base + Cfg::kEmpty2;
            const uint32_t full2_leader = ptx::mapa(full2, 0);
            const int rb = row_b + unit_half(cur) * Cfg::kMmaN;  // the 256-column block of B
            for (int kb = cur.kb_begin; kb < cur.kb_end; ++kb) {
              if (!ptx::mbar_wait(empty2 + 8 * hstage, hphase ^ 1u, wd, kSiteProducer, t)) {
                ok = false;
                break;
              }
              if (leader) ptx::mbar_arrive_expect_tx(full2 + 8 * hstage, 2u * Cfg::kHalfStageBytes);
              const uint32_t fb = full2_leader + 8 * hstage;
              const uint32_t dst = sA + hstage * Cfg::kHalfStageBytes;
              ptx::tma_load_2d_cg2(dst, &map_a, fb, kb * kBlockK, row_a, policy_a);
              ptx::tma_load_2d_cg2(dst + kStageBytesA, &map_b, fb, kb * kBlockK, rb, policy_b);
              if (++hstage == static_cast<uint32_t>(Cfg::kHalfStages)) {
                hstage = 0;
                hphase ^= 1u;
              }
            }
            continue;
          }
        }
        for (int kb = cur.kb_begin; kb < cur.kb_end; ++kb) {
          if (!ptx::mbar_wait(empty0 + 8 * stage, phase ^ 1u, wd, kSiteProducer, t)) {
            ok = false;
            break;
          }
          if (leader) ptx::mbar_arrive_expect_tx(full0 + 8 * stage, Cfg::kTxBytes);
          const uint32_t fb = full_leader0 + 8 * stage;
          ptx::tma_load_2d_cg2(sA + stage * kStageBytesA, &map_a, fb, kb * kBlockK, row_a, policy_a);
#pragma unroll
          for (int h = 0; h < NB; ++h) {
            ptx::tma_load_2d_cg2(sB + stage * Cfg::kStageBytesB + h * Cfg::kBlockBytesB, &map_b, fb,
                                 kb * kBlockK, row_b + h * Cfg::kMmaN, policy_b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
    if (p.pdl != kPdlOff) ptx::griddep_launch_dependents();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (leader && lane == 0) {
      const uint32_t own_empty0 = ptx::mapa(empty0, 0), peer_empty0 = ptx::mapa(empty0, 1);
      const uint32_t own_tfull0 = ptx::mapa(tfull0, 0), peer_tfull0 = ptx::mapa(tfull0, 1);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      [[maybe_unused]] uint32_t hstage = 0, hphase = 0;
      bool ok = true;
      for (uint32_t t = cluster; t < num_units && ok; t += nclusters) {
        const WorkUnit cur = unit_at<Cfg::kHalfTail>(p, t);
        if (!ptx::mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1u, wd, kSiteMmaTmemEmpty, t)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccStride;
        if constexpr (Cfg::kHalfTail) {
          if (cur.slot <= -2) {
            // Half unit: the re-cut ring, one N = 256 MMA per K step into
            // TMEM columns 0..255.
            const uint32_t full2 = base + Cfg::kFull2, empty2 = base + Cfg::kEmpty2;
            const uint32_t own_empty2 = ptx::mapa(empty2, 0), peer_empty2 = ptx::mapa(empty2, 1);
            for (int kb = cur.kb_begin; kb < cur.kb_end; ++kb) {
              if (!ptx::mbar_wait(full2 + 8 * hstage, hphase, wd, kSiteMmaFull, t)) {
                ok = false;
                break;
              }
              ptx::tc_fence_after();
              const uint32_t src = sA + hstage * Cfg::kHalfStageBytes;
              const uint64_t a_desc = smem_desc(src);
              const uint64_t b_desc = smem_desc(src + kStageBytesA);
#pragma unroll
              for (int k = 0; k < kBlockK / kMmaK; ++k) {
                ptx::mma_bf16_cg2(d_tmem, a_desc + 2 * k, b_desc + 2 * k, Cfg::kIdesc,
                                  (kb > cur.kb_begin || k > 0) ? 1u : 0u);
              }
              ptx::mma_commit_cg2(own_empty2 + 8 * hstage);
              ptx::mma_commit_cg2(peer_empty2 + 8 * hstage);
              if (++hstage == static_cast<uint32_t>(Cfg::kHalfStages)) {
                hstage = 0;
                hphase ^= 1u;
              }
            }
            if (!ok) break;
            ptx::mma_commit_cg2(own_tfull0 + 8 * acc);
            ptx::mma_commit_cg2(peer_tfull0 + 8 * acc);
            if (++acc == Cfg::kAccBufs) {
              acc = 0;
              acc_phase ^= 1u;
            }
            continue;
          }
        }
        for (int kb = cur.kb_begin; kb < cur.kb_end; ++kb) {
          if (!ptx::mbar_wait(full0 + 8 * stage, phase, wd, kSiteMmaFull, t)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint64_t a_desc = smem_desc(sA + stage * kStageBytesA);
          const uint64_t b_desc = smem_desc(sB + stage * Cfg::kStageBytesB);
#pragma unroll
          for (int k = 0; k < kBlockK / kMmaK; ++k) {
#pragma unroll
            for (int h = 0; h < NB; ++h) {
              // +32 bytes per K step inside the 128-byte swizzle row; the
              // second N block of B sits kBlockBytesB further on.
              ptx::mma_bf16_cg2(d_tmem + h * Cfg::kMmaN, a_desc + 2 * k,
                                b_desc + (h * Cfg::kBlockBytesB >> 4) + 2 * k, Cfg::kIdesc,
                                (kb > cur.kb_begin || k > 0) ? 1u : 0u);
            }
          }
          ptx::mma_commit_cg2(own_empty0 + 8 * stage);
          ptx::mma_commit_cg2(peer_empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::mma_commit_cg2(own_tfull0 + 8 * acc);
        ptx::mma_commit_cg2(peer_tfull0 + 8 * acc);
        if (++acc == Cfg::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA this thread issued must be complete before TMEM is freed
      // and before the peer CTA (whose shared memory the MMAs read) exits.
      ptx::mma_commit_cg2(ptx::mapa(drain, 0));
      ptx::Watchdog dwd = wd;
      dwd.timeout_ns = 100000000ull;  // 100 ms: independent of the caller's budget
      ptx::mbar_wait_drain(drain, 0, dwd, kSiteDrain);
    }
    __syncwarp();
    if (p.pdl != kPdlOff) ptx::griddep_launch_dependents();
  } else {
    // ------------------------------------------------------------ epilogue
    const uint32_t e = warp - 2u;         // epilogue warp index
    const uint32_t quarter = warp & 3u;   // TMEM lanes this warp may access
    const uint32_t nblk = e >> 2;         // which slice of kColsPerWarp columns of the tile
    const uint32_t cstage0 = sC + e * Cfg::kCBufs * kCStageBytes;
    const uint32_t tempty_leader0 = ptx::mapa(tempty0, 0);
    uint32_t acc = 0, acc_phase = 0, cbuf = 0;
    const uint32_t ticket = base + Cfg::kTicket;
    WorkUnit nxt = (cluster < num_units) ? unit_at<Cfg::kHalfTail>(p, cluster) : WorkUnit{0, 0, 0, -1};
    for (uint32_t t = cluster; t < num_units; t += nclusters) {
      const WorkUnit cur = nxt;
      if (t + nclusters < num_units) nxt = unit_at<Cfg::kHalfTail>(p, t + nclusters);
      const uint32_t tile = cur.tile;
      const int row = static_cast<int>(tile >> 16) * kTileM + static_cast<int>(rank) * 128 +
                      static_cast<int>(quarter) * 32;
      // A half unit's accumulator is TMEM columns 0..255 for global columns
      // half * 256 ..; the warps holding columns 256..511 have nothing.
      const int half = Cfg::kHalfTail ? unit_half(cur) : -1;
      const int half_off = half >= 0 ? half * Cfg::kMmaN : 0;
      const bool idle_half = half >= 0 && static_cast<int>(nblk) * Cfg::kColsPerWarp >= Cfg::kMmaN;
      const int col0 = static_cast<int>(tile & 0xFFFFu) * Cfg::kTileN + half_off +
                       static_cast<int>(nblk) * Cfg::kColsPerWarp;
      [[maybe_unused]] uint32_t bias_w[4];
      [[maybe_unused]] uint32_t res_w[16];
      if constexpr (Cfg::kEpi) {
        const int r = row + static_cast<int>(lane);
        if ((p.epi_flags & kEpiResidual) && r < p.M) {
          // This lane's residual row for the whole column block, into L2 while
          // the MMAs run, so the per-chunk loads below wait on L2, not DRAM.
          const uint16_t* src = p.residual + static_cast<long long>(r) * p.ldr;
#pragma unroll
          for (int b = 1; b < (Cfg::kColsPerWarp * 2 + 127) / 128; ++b)
            if (col0 + 64 * b < p.N) ptx::prefetch_l2(src + col0 + 64 * b);
        }
        epi_load_bias(p, col0, Cfg::kColsPerWarp, lane, bias_w);
        epi_load_residual(p, r, col0, res_w);
      }
      // After a timeout (here or in another role) the loop keeps running
      // without doing work, so every epilogue warp still reaches every named
      // barrier of the K-slice path below; later waits fail immediately.
      const bool full_ok = ptx::mbar_wait(tfull0 + 8 * acc, acc_phase, wd, kSiteEpilogue, t);
      const bool live = __all_sync(0xFFFFFFFFu, full_ok);  // warp-uniform
      ptx::tc_fence_after();
      // The last accumulator is complete: the next kernel may start its setup.
      if (p.pdl != kPdlOff && t + nclusters >= num_units) ptx::griddep_launch_dependents();
      const uint32_t t_row =
          tmem_base + ((quarter * 32u) << 16) + acc * Cfg::kAccStride + nblk * Cfg::kColsPerWarp;
      if (cur.slot < 0 && !live) {
        // nothing to do for this tile
      } else if (idle_half) {
        // Columns this warp would drain belong to no tile in a half unit.
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(tempty_leader0 + 8 * acc);
      } else if (cur.slot < 0) {
        // Whole tile: chunks of 32 columns: TMEM -> registers -> bf16 ->
        // swizzled staging buffer -> TMA store, two buffers in flight per warp.
        auto tmem_chunk = [&](int c, uint32_t (&v)[32]) {
          ptx::tmem_ld_32x32b_x32(t_row + c * kCBoxCols, v);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v);
          if (c == Cfg::kWarpChunks - 1) {
            // This warp's part of the accumulator is in registers: release it.
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_cluster(tempty_leader0 + 8 * acc);
          }
        };
        auto store_bf16 = [&](int c, const uint32_t (&v)[32]) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = ptx::pack_bf16x2(v[2 * i], v[2 * i + 1]);
          store_c_chunk<Cfg>(pk, col0 + c * kCBoxCols, row, lane, cstage0, cbuf, map_c, p);
        };
        if constexpr (Cfg::kEpi) {
          // The residual of chunk c + 1 loads while chunk c is finished; two
          // buffers take turns so no register copy waits on those loads.
          uint32_t res_b[16];
          auto chunk = [&](int c, const uint32_t (&cur)[16], uint32_t (&nxt)[16]) {
            if (c + 1 < Cfg::kWarpChunks)
              epi_load_residual(p, row + static_cast<int>(lane), col0 + (c + 1) * kCBoxCols, nxt);
            uint32_t v[32];
            tmem_chunk(c, v);
            apply_epilogue(v, c, bias_w, cur, p);
            if (p.out_type == kOutE4m3) {
              uint32_t q8[8];
#pragma unroll
              for (int i = 0; i < 8; ++i)
                q8[i] = ptx::pack_e4m3x4(p.out_scale * __uint_as_float(v[4 * i]),
                                         p.out_scale * __uint_as_float(v[4 * i + 1]),
                                         p.out_scale * __uint_as_float(v[4 * i + 2]),
                                         p.out_scale * __uint_as_float(v[4 * i + 3]));
              store_e4m3_row(q8, row + static_cast<int>(lane), col0 + c * kCBoxCols, p);
            } else if (p.out_type == kOutF32) {
              uint32_t lo[16], hi[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                lo[i] = v[i];
                hi[i] = v[16 + i];
              }
              const int col = col0 + c * kCBoxCols;
              store_c_chunk<Cfg, 4>(lo, col, row, lane, cstage0, cbuf, map_c, p);
              store_c_chunk<Cfg, 4>(hi, col + 16, row, lane, cstage0, cbuf, map_c, p);
            } else {
              store_bf16(c, v);
            }
          };
#pragma unroll 1
          for (int c = 0; c < Cfg::kWarpChunks; c += 2) {
            chunk(c, res_w, res_b);
            if (c + 1 < Cfg::kWarpChunks) chunk(c + 1, res_b, res_w);
          }
        } else if constexpr (Cfg::kStagedDrain) {
          // One accumulator for the whole tile: the next tile's MMAs wait
          // until every warp has read its part, and those reads are bound by
          // the SM's TMEM read rate (about 1.1 us for 256 KB).  So a warp
          // reads all its chunks before any store, two loads in flight at a
          // time: the first kCBufs go to its staging buffers, the others stay
          // in registers as packed bf16; then it releases the accumulator and
          // issues the TMA stores.  A slice that reaches past M or N takes the
          // per-chunk path below.
          constexpr int kStaged = Cfg::kCBufs, kHeld = Cfg::kHeldChunks;
          const bool whole = row < p.M && col0 + Cfg::kColsPerWarp <= p.N;
          if (whole) {
            if (lane == 0) ptx::bulk_wait_group_read<0>();  // the previous tile's stores have read every buffer
            __syncwarp();
#pragma unroll
            for (int c = 0; c < kStaged; c += 2) {
              uint32_t v0[32], v1[32];
              ptx::tmem_ld_32x32b_x32(t_row + c * kCBoxCols, v0);
              if (c + 1 < kStaged) ptx::tmem_ld_32x32b_x32(t_row + (c + 1) * kCBoxCols, v1);
              ptx::tmem_wait_ld();
              ptx::reg_fence32(v0);
              stage_chunk_row_f32(cstage0 + c * kCStageBytes, lane, v0);
              if (c + 1 < kStaged) {
                ptx::reg_fence32(v1);
                stage_chunk_row_f32(cstage0 + (c + 1) * kCStageBytes, lane, v1);
              }
            }
            uint32_t pk[kHeld][16];
#pragma unroll
            for (int h = 0; h < kHeld; h += 2) {
              uint32_t v0[32], v1[32];
              ptx::tmem_ld_32x32b_x32(t_row + (kStaged + h) * kCBoxCols, v0);
              if (h + 1 < kHeld) ptx::tmem_ld_32x32b_x32(t_row + (kStaged + h + 1) * kCBoxCols, v1);
              ptx::tmem_wait_ld();
              ptx::reg_fence32(v0);
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[h][i] = ptx::pack_bf16x2(v0[2 * i], v0[2 * i + 1]);
              if (h + 1 < kHeld) {
                ptx::reg_fence32(v1);
#pragma unroll
                for (int i = 0; i < 16; ++i) pk[h + 1][i] = ptx::pack_bf16x2(v1[2 * i], v1[2 * i + 1]);
              }
            }
            // Every TMEM read of this warp is done: release the accumulator.
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_cluster(tempty_leader0 + 8 * acc);
            if (p.mc_c != nullptr) {
              __syncwarp();
#pragma unroll 1
              for (int c = 0; c < kStaged; ++c)
                copy_chunk_to_multicast<2>(cstage0 + c * kCStageBytes, col0 + c * kCBoxCols, row, lane, p);
              __syncwarp();
            } else {
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
#pragma unroll
                for (int c = 0; c < kStaged; ++c) {
                  ptx::tma_store_2d(&map_c, cstage0 + c * kCStageBytes, col0 + c * kCBoxCols, row);
                  ptx::bulk_commit_group();
                }
              }
              if (p.npeers > 0) {
#pragma unroll 1
                for (int c = 0; c < kStaged; ++c)
                  copy_chunk_to_peers<2>(cstage0 + c * kCStageBytes, col0 + c * kCBoxCols, row, lane, p);
              }
            }
            cbuf = 0;  // held chunk h reuses buffer h % kCBufs once the store before it there has read it
#pragma unroll
            for (int h = 0; h < kHeld; ++h)
              store_c_chunk<Cfg>(pk[h], col0 + (kStaged + h) * kCBoxCols, row, lane, cstage0, cbuf, map_c, p);
          } else {
#pragma unroll 1
            for (int c = 0; c < Cfg::kWarpChunks; ++c) {
              uint32_t v[32];
              tmem_chunk(c, v);  // releases the accumulator after the last chunk's read
              store_bf16(c, v);
            }
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < Cfg::kWarpChunks; ++c) {
            uint32_t v[32];
            tmem_chunk(c, v);
            store_bf16(c, v);
          }
        }
      } else if constexpr (Cfg::kTailSplit) {
        // K slice of a split tile.  Partials are laid out so that the 32
        // threads of a warp (32 consecutive rows) touch 512 contiguous bytes
        // per 16-byte column group: [column group][row 0..127] of float4.
        const uint32_t i = quarter * 32u + lane;  // row of this CTA's 128
        const int tile_r = cur.slot / p.tail_split;
        const size_t slab = static_cast<size_t>(128) * Cfg::kTileN;  // floats per CTA per slice
        auto part = [&](int slot) { return p.workspace + (static_cast<size_t>(slot) * 2 + rank) * slab; };
        float* mine = part(cur.slot);
#pragma unroll 1
        for (int c = 0; c < (live ? Cfg::kWarpChunks : 0); ++c) {
          uint32_t v[32];
          ptx::tmem_ld_32x32b_x32(t_row + c * kCBoxCols, v);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const size_t g = static_cast<size_t>((nblk * (Cfg::kWarpChunks) + c) * 8 + j);
            ptx::st_global_v4(mine + (g * 128 + i) * 4, v[4 * j], v[4 * j + 1], v[4 * j + 2],
                              v[4 * j + 3]);
          }
        }
        // Ticket: the last K slice of this half-tile finishes it.
        __threadfence();
        ptx::named_barrier(1, 32 * Cfg::kEpiWarps);
        if (threadIdx.x == 64) {
          uint32_t last = 0u;
          if (!ptx::aborted(wd)) {
            const unsigned int old = atomicAdd(&p.tail_counters[tile_r * 2 + rank], 1u);
            last = (old == static_cast<unsigned int>(p.tail_split - 1)) ? 1u : 0u;
            if (last) p.tail_counters[tile_r * 2 + rank] = 0u;  // ready for the next launch
          }
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(ticket), "r"(last) : "memory");
        }
        ptx::named_barrier(1, 32 * Cfg::kEpiWarps);
        uint32_t is_last;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(is_last) : "r"(ticket) : "memory");
        if (is_last && !ptx::aborted(wd)) {
          __threadfence();
          const int first = tile_r * p.tail_split;
#pragma unroll 1
          for (int c = 0; c < Cfg::kWarpChunks; ++c) {
            // Sum the slices in slice order whichever slice arrives last, so
            // the result does not depend on timing; this slice's own partial
            // comes from TMEM at its place in the order.  Two 16-column halves
            // keep the registers in check.
            uint32_t pk[16];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              float acc16[16];
#pragma unroll 1
              for (int sl = 0; sl < p.tail_split; ++sl) {
                float x[16];
                if (first + sl == cur.slot) {
                  uint32_t v[16];
                  ptx::tmem_ld_32x32b_x16(t_row + c * kCBoxCols + hh * 16, v);
                  ptx::tmem_wait_ld();
                  ptx::reg_fence16(v);
#pragma unroll
                  for (int k = 0; k < 16; ++k) x[k] = __uint_as_float(v[k]);
                } else {
                  const float* other = part(first + sl);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const size_t g =
                        static_cast<size_t>((nblk * (Cfg::kWarpChunks) + c) * 8 + hh * 4 + j);
                    uint32_t x0, x1, x2, x3;
                    ptx::ld_global_cg_v4(other + (g * 128 + i) * 4, x0, x1, x2, x3);
                    x[4 * j] = __uint_as_float(x0);
                    x[4 * j + 1] = __uint_as_float(x1);
                    x[4 * j + 2] = __uint_as_float(x2);
                    x[4 * j + 3] = __uint_as_float(x3);
                  }
                }
#pragma unroll
                for (int k = 0; k < 16; ++k) acc16[k] = (sl == 0) ? x[k] : acc16[k] + x[k];
              }
#pragma unroll
              for (int k = 0; k < 8; ++k)
                pk[hh * 8 + k] = ptx::pack_bf16x2(__float_as_uint(acc16[2 * k]),
                                                  __float_as_uint(acc16[2 * k + 1]));
            }
            store_c_chunk<Cfg>(pk, col0 + c * kCBoxCols, row, lane, cstage0, cbuf, map_c, p);
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(tempty_leader0 + 8 * acc);
      }
      if (++acc == Cfg::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) ptx::bulk_wait_group_read<0>();  // staging reusable; the stores land before the kernel completes
    if (p.npeers > 0 || p.mc_c != nullptr) __threadfence_system();  // peer copies visible before the kernel ends
    __syncwarp();
  }

  // --------------------------------------------------------------- teardown
  if (threadIdx.x == 0 && ptx::aborted(wd)) {
    // Let TMA loads that were issued but never consumed land before exit.
    ptx::sleep_ns_bounded(200000ull);
  }
  ptx::tc_fence_before();
  ptx::cluster_sync_all();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc_cg2(tmem_base, kTmemCols);
}

// Self-test of the watchdog: every CTA waits on an mbarrier that nothing
// ever arrives on.  The bounded wait must give up after `timeout_ns`, record
// kStatusTimeout and let the kernel exit normally.
__global__ void __launch_bounds__(32, 1) __cluster_dims__(2, 1, 1)
    watchdog_selftest_kernel(unsigned int* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_word;
  const uint32_t rank = ptx::cluster_ctarank();
  ptx::Watchdog wd;
  wd.abort_flag = ptx::smem_u32(&abort_word);
  wd.peer_abort_flag = ptx::mapa(wd.abort_flag, rank ^ 1u);
  wd.status = status;
  wd.timeout_ns = timeout_ns;
  if (threadIdx.x == 0) {
    abort_word = 0;
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    ptx::fence_mbar_init_cluster();
  }
  ptx::cluster_sync_all();
  if (threadIdx.x == 0) {
    ptx::mbar_wait(ptx::smem_u32(&bar), 0, wd, kSiteSelftest, 0);
  }
  __syncwarp();
  ptx::cluster_sync_all();
}

}  // namespace b200gemm
