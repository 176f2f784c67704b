// Host side of the C-ABI in include/b200gemm.h: argument validation, the
// per-handle caches (tensor maps, tile schedules), device status words and
// kernel launches.  Replaces the reference launcher runKernel1
// (b200_kernels/matmul_1.cuh:386-418) and its hidden globals (:5-11).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "b200gemm.h"
#include "gemm_decode_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_smallm1_sm100.cuh"
#include "schedule.cuh"

namespace b200gemm {

// Pipeline depth of each kernel instance (build-time tuning knobs).
#ifndef B200GEMM_STAGES_N256
#define B200GEMM_STAGES_N256 6
#endif
#ifndef B200GEMM_STAGES_N512
#define B200GEMM_STAGES_N512 3
#endif
#ifndef B200GEMM_EPIWARPS_N512
#define B200GEMM_EPIWARPS_N512 8
#endif
// L2 sector promotion of every tensor map's loads (CUtensorMapL2promotion:
// 0 none, 1 64 B, 2 128 B, 3 256 B).
#ifndef B200GEMM_L2_PROMOTION
#define B200GEMM_L2_PROMOTION 3
#endif
// Small-M pair kernel over 128- or 256-row blocks of A for small shapes of up
// to this many rows (256 = never above 256 rows).
#ifndef B200GEMM_SMALLM_MAX_ROWS
#define B200GEMM_SMALLM_MAX_ROWS 4096
#endif
// Small-M pair kernel: allow a K split over 3 CTA pairs (129..256 rows of A).
#ifndef B200GEMM_SMALLM_SPLIT3
#define B200GEMM_SMALLM_SPLIT3 1
#endif
// Time of a 256 x 448 tile relative to a 256 x 512 tile in the width model.
#ifndef B200GEMM_TILE448_SCALE
#define B200GEMM_TILE448_SCALE 0.9
#endif
#ifndef B200GEMM_DEFAULT_ORDER
#define B200GEMM_DEFAULT_ORDER 1
#endif
#ifndef B200GEMM_DEFAULT_BAND
#define B200GEMM_DEFAULT_BAND 16
#endif
using CfgN256 = GemmCfg<B200GEMM_STAGES_N256, 1>;  // 256 x 256 tiles, overlapped epilogue
// 256 x 512 tiles, shared A stage; 8 epilogue warps drain the single
// 512-column accumulator, each reading its 8 chunks into 4 staging buffers
// and registers before any store (3 stages leave room for the buffers; 8
// warps leave 160+ registers per thread, so nothing spills).
using CfgN512 = GemmCfg<B200GEMM_STAGES_N512, 2, 256, false, B200GEMM_EPIWARPS_N512>;
// The same tiles, launched only when a short last wave runs as 256-column halves.
using CfgN512H = GemmCfg<B200GEMM_STAGES_N512, 2, 256, false, B200GEMM_EPIWARPS_N512, true>;
// 256 x 448 tiles (two N = 224 MMAs per K step sharing the A stage), so a
// shared-A tile also divides N = 1792 (the 8-way shard of N = 14336), and
// their half-width form for a short last wave.
using CfgN448 = GemmCfg<B200GEMM_STAGES_N512, 2, 224, false, B200GEMM_EPIWARPS_N512>;
using CfgN448H = GemmCfg<B200GEMM_STAGES_N512, 2, 224, false, B200GEMM_EPIWARPS_N512, true>;
// Narrower tiles for N that 256 does not divide into full waves (e.g. an
// N-sharded projection with N = 1792 = 8 x 224); more stages fit because each
// stage holds fewer B rows.
using CfgN224 = GemmCfg<6, 1, 224>;
using CfgN192 = GemmCfg<7, 1, 192>;
using CfgN128 = GemmCfg<8, 1, 128>;
// The same five widths with the fused epilogue compiled in.
using CfgE256 = GemmCfg<B200GEMM_STAGES_N256, 1, 256, true>;
#ifndef B200GEMM_STAGES_E512
#define B200GEMM_STAGES_E512 4
#endif
using CfgE512 = GemmCfg<B200GEMM_STAGES_E512, 2, 256, true>;  // 8 epilogue warps: the fused math needs their registers
using CfgE448 = GemmCfg<B200GEMM_STAGES_E512, 2, 224, true>;
using CfgE224 = GemmCfg<6, 1, 224, true>;
using CfgE192 = GemmCfg<7, 1, 192, true>;
using CfgE128 = GemmCfg<8, 1, 128, true>;
// Tile widths of the tiled kernel, in the order the cost model prefers them
// on a tie; index i of every per-width table below.
constexpr int kWidths[] = {256, 512, 448, 224, 192, 128};
constexpr int kNumWidths = 6;
inline int width_index(int width) {
  for (int i = 0; i < kNumWidths; ++i)
    if (kWidths[i] == width) return i;
  return -1;
}
constexpr int kVersion = 10000;  // 1.0.0
constexpr int kMapCacheSize = 32;   // the host-staged path uses one entry per row chunk
constexpr size_t kScheduleCacheSize = 16;
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;
constexpr int kMaxTailCounters = 1024;   // two per split tile (one per CTA of the pair)
constexpr int kMaxTailSplit = 6;

// K split of the last, partial wave.  With T tiles on G clusters the last
// wave has R = T mod G tiles and leaves G - R clusters idle; splitting each
// of those tiles into S K slices (R * S <= G, at least 4 K blocks per slice,
// S <= kMaxTailSplit because the last slice reads the other S - 1 partials)
// shortens that wave to about 1/S of a tile.  Returns S (1 = no split).
int tail_split_for(int tiles, int clusters, int num_kb) {
  const int rem = tiles % clusters;  // a single partial wave is all tail
  if (rem == 0) return 1;
  int sk = clusters / rem;
  if (sk > kMaxTailSplit) sk = kMaxTailSplit;
  if (sk > num_kb / 4) sk = num_kb / 4;
  while (sk >= 2) {
    const int per = (num_kb + sk - 1) / sk;
    if ((sk - 1) * per < num_kb) break;  // no empty slice
    --sk;
  }
  return sk >= 2 ? sk : 1;
}

// Restores the caller's current device on scope exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    ok_ = cudaGetDevice(&prev_) == cudaSuccess;
    if (ok_ && prev_ != device) ok_ = cudaSetDevice(device) == cudaSuccess;
    switched_ = ok_ && prev_ != device;
  }
  ~DeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = false;
  bool switched_ = false;
};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// Row-major matrix [outer x inner] (bf16 unless `dtype` says otherwise) with a row pitch in bytes, read or
// written in boxes of [box_outer x box_inner] through a shared-memory swizzle.
bool encode_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer,
               uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle,
               CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r =
      encode(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box,
             elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             static_cast<CUtensorMapL2promotion>(B200GEMM_L2_PROMOTION), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct MapEntry {
  bool valid = false;
  const void* a = nullptr;
  const void* b = nullptr;
  void* c = nullptr;
  int M = 0, N = 0, K = 0, ldc = 0;
  int b_rows = 0;   // rows of B's box: B rows one CTA loads per MMA column block
  int c_type = 0;   // C element type (fused epilogue output type, B200GEMM_OUT_*)
  uint64_t last_use = 0;
  CUtensorMap map_a, map_b, map_c;
};

struct ScheduleEntry {
  uint32_t tiles_m = 0, tiles_n = 0;
  int order = 0;
  uint32_t band = 0;
  uint32_t* dev = nullptr;
  uint64_t last_use = 0;
};

// Opt the kernel instance into its shared memory size and return how many
// of its 2-CTA clusters fit on the device at once (0 on failure).
template <class Cfg>
int prepare_kernel(int sm_count) {
  if (cudaFuncSetAttribute(gemm_bf16_nt_sm100<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           Cfg::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(sm_count & ~1), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_bf16_nt_sm100<Cfg>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

// Small-M instances (K split over 1, 2 or 4 CTA pairs of one cluster).
template <class Cfg>
int prepare_decode_kernel(int sm_count) {
  if (cudaFuncSetAttribute(gemm_bf16_nt_decode_sm100<Cfg>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (Cfg::kClusterSize > 8 &&
      cudaFuncSetAttribute(gemm_bf16_nt_decode_sm100<Cfg>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                           1) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  // Clusters of 2S CTAs that fit on the device at once: fewer than
  // sm_count / 2S, since a cluster must sit inside one GPC.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Cfg::kClusterSize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(sm_count / Cfg::kClusterSize * Cfg::kClusterSize), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_bf16_nt_decode_sm100<Cfg>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

// Same for the single-CTA small-M kernel (clusters of S CTAs).
template <class Cfg>
int prepare_smallm1_kernel(int sm_count) {
  if (cudaFuncSetAttribute(gemm_bf16_nt_smallm1_sm100<Cfg>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Cfg::kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(sm_count / Cfg::kSplit * Cfg::kSplit), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_bf16_nt_smallm1_sm100<Cfg>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

template <class Cfg>
cudaError_t launch_smallm1(cudaStream_t stream, const CUtensorMap& ma, const CUtensorMap& mb,
                           const CUtensorMap& mc, const CUtensorMap& mr, const SmallMParams& p) {
  const unsigned clusters = static_cast<unsigned>((p.N + 127) / 128);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Cfg::kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(clusters * Cfg::kSplit, 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.pdl != kPdlOff) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, gemm_bf16_nt_smallm1_sm100<Cfg>, ma, mb, mc, mr, p);
}

template <class Cfg>
cudaError_t launch_decode(cudaStream_t stream, const CUtensorMap& ma, const CUtensorMap& mb,
                          const CUtensorMap& mc, const CUtensorMap& mr, const DecodeParams& p) {
  const unsigned clusters =
      static_cast<unsigned>(p.n_blocks) * static_cast<unsigned>((p.M + Cfg::kNT - 1) / Cfg::kNT);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Cfg::kClusterSize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(clusters * Cfg::kClusterSize, 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.pdl != kPdlOff) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, gemm_bf16_nt_decode_sm100<Cfg>, ma, mb, mc, mr, p);
}

template <class Cfg>
cudaError_t launch_gemm(int clusters, cudaStream_t stream, const CUtensorMap& ma,
                        const CUtensorMap& mb, const CUtensorMap& mc, const GemmParams& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (p.pdl != kPdlOff) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemm_bf16_nt_sm100<Cfg>, ma, mb, mc, p);
}

// Relative cost of a GEMM with tiles `width` columns wide: waves of
// persistent clusters times the time of one tile, in units of one 64-deep K
// block of a 256 x 256 tile at full tensor rate.  Tiles up to 256 wide are
// bound by the operand bytes each SM pulls from L2 per K block (A 16 KB plus
// width / 2 B rows of 128 B), so their time follows those bytes rather than
// the flops: measured on B200, tiles of 224, 192 and 128 columns take 0.95,
// 0.89 and 0.785 of a 256-wide tile's time (0.875, 0.75 and 0.5 of its
// flops), fitted as 0.08 + 0.92 x bytes / 32 KB, at 0.85 tensor efficiency
// for 256.  The 512-wide tile shares one A stage between two MMAs and pays
// its non-overlapped epilogue; fitted on 8192^3 and 16384 x 14336 x 4096
// (where 512 wins by 9.8% and 1.3%): its K blocks run 1 / 0.8545 as fast
// per flop as the 256-wide tile's and the epilogue costs 13 K blocks (17
// before the accumulator read-out went ahead of the stores; with 13,
// 16384 x 2048 x 4096 moves to 512-wide tiles, measured 2% faster).
// `epi` adds the fused epilogue's measured per-tile cost (epilogue_cost).
double tile_plan_cost(int width, uint32_t tiles_m, int N, int num_kb, int clusters,
                      double epi = 0.0, bool half_tail = false) {
  if (clusters <= 0) return 1e300;
  const uint64_t tiles_n = (static_cast<uint64_t>(N) + width - 1) / width;
  const uint64_t tiles = tiles_m * tiles_n;
  const uint64_t waves = (tiles + clusters - 1) / clusters;
  auto narrow_time = [&](int w) {
    const double feed = (16384.0 + 64.0 * w) / 32768.0;
    return num_kb * (0.08 + 0.92 * feed) / 0.85;
  };
  if (width == 512 || width == 448) {
    // 448: two N = 224 MMAs and 7/8 of the read-out per tile.
    const double scale = width == 448 ? B200GEMM_TILE448_SCALE : 1.0;
    const double tile_time = scale * (2.0 * num_kb + 13.0) * 0.8545 / 0.85;
    const uint64_t rem = tiles % static_cast<uint64_t>(clusters);
    if (half_tail && epi == 0.0 && rem > 0 && 2 * rem <= static_cast<uint64_t>(clusters)) {
      // The last wave runs as 256-column halves on their own 4-stage ring:
      // about 0.45-0.65 of a whole tile's cycles in ncu captures; 0.6 here.
      return (static_cast<double>(waves - 1) + 0.6) * tile_time;
    }
    return static_cast<double>(waves) * (tile_time + epi);
  }
  return static_cast<double>(waves) * (narrow_time(width) + epi);
}

// Per-tile cost of a fused epilogue, in tile_plan_cost's units, measured on
// B200 at 8192^3 and 16384 x 14336 x 4096 (constant in K): the 512-wide
// tile pays it in full (its epilogue is not overlapped with MMAs), a 256-wide
// tile about a third (its epilogue overlaps the next tile's MMAs), narrower
// tiles in proportion to their columns.
double epilogue_cost(const b200gemm_epilogue* epi, int width) {
  if (epi == nullptr) return 0.0;
  double w512 = 0.0, w256 = 0.0;
  switch (epi->activation) {
    case B200GEMM_ACT_RELU: w512 = 8.0; w256 = 2.5; break;
    case B200GEMM_ACT_GELU_TANH: w512 = 14.0; w256 = 5.0; break;
    case B200GEMM_ACT_GELU: w512 = 28.0; w256 = 10.0; break;
    case B200GEMM_ACT_SILU: w512 = 16.0; w256 = 4.6; break;
    default: break;
  }
  if (epi->residual != nullptr) {
    w512 += 16.0;
    w256 += 6.0;
  }
  if (epi->bias != nullptr && epi->activation == B200GEMM_ACT_NONE && epi->residual == nullptr) {
    w512 += 6.0;
    w256 += 2.2;
  }
  if (epi->out_type == B200GEMM_OUT_F32) {
    w512 += 12.0;
    w256 += 4.0;
  } else if (epi->out_type == B200GEMM_OUT_E4M3) {
    w512 += 2.0;
    w256 += 0.5;
  }
  if (width == 512 || width == 448) return w512 * width / 512.0;
  return w256 * width / 256.0;
}

}  // namespace b200gemm

using namespace b200gemm;

// Device buffers, streams and events of b200gemm_bf16_nt_host (created on
// first use, grown when a larger problem arrives).  Consecutive calls
// alternate between two buffer sets, so a call's uploads start as soon as the
// previous call's uploads end, while that call's last GEMM and copy-out
// still run; a set is reused only after the call two back has finished with
// it.
struct HostStaging {
  struct Buffers {
    void* dA = nullptr;
    void* dB = nullptr;
    void* dC = nullptr;
    size_t capA = 0, capB = 0, capC = 0;
    cudaEvent_t ev_read = nullptr;  // last GEMM of the last call on this set: dA, dB free
    cudaEvent_t ev_done = nullptr;  // last copy-out of that call: dC free
  };
  Buffers set[2];
  int next = 0;
  bool ready = false;
  cudaStream_t s_h2d = nullptr, s_mma = nullptr, s_d2h = nullptr;
  static constexpr int kMaxChunks = 16;
  cudaEvent_t ev_start = nullptr, ev_b = nullptr;
  cudaEvent_t ev_a[kMaxChunks] = {}, ev_c[kMaxChunks] = {};
};

struct b200gemm_handle {
  int device = 0;
  int sm_count = 0;
  int max_clusters = 0;       // co-resident 2-CTA clusters (the smaller of the two instances)
  int clusters_w[kNumWidths] = {};  // co-resident clusters of each width's instance
  int clusters_epi[kNumWidths] = {};  // the same for the fused-epilogue instances
  int decode_clusters[5] = {};        // [S]: co-resident clusters of the small-M pair kernel, split S
  int decode256_clusters[5] = {};     // the same for its instances covering 256 rows of A
  int smallm1_clusters[5] = {};       // [S]: the same for the single-CTA small-M kernel
  int tile_width = 0;         // 0 = choose per call, else one of kWidths
  int small_m = -1;           // small-M kernel: -1 or 1 = use it when eligible, 0 = never
  int pdl = 0;                // B200GEMM_PDL_*: launch overlap with the previous kernel
  unsigned int* status_dev = nullptr;
  unsigned long long timeout_ns = kDefaultTimeoutNs;
  int order = B200GEMM_DEFAULT_ORDER;      // tile order (schedule.cuh)
  uint32_t band = B200GEMM_DEFAULT_BAND;   // tile-rows per band for the band order
  std::mutex mu;
  uint64_t tick = 0;
  MapEntry maps[kMapCacheSize];
  HostStaging staging;
  // K-split tail: fp32 partials of the last wave's split tiles and their
  // tickets (zeroed once; the kernel resets each ticket after use).  Split
  // launches share them, so each waits for the previous one (tail_event).
  float* tail_ws = nullptr;
  size_t tail_ws_bytes = 0;
  unsigned int* tail_counters = nullptr;
  cudaEvent_t tail_event = nullptr;
  bool tail_event_recorded = false;
  bool tail_split_enabled = false;  // off by default until its reduction beats the idle wave
  bool tail_half_enabled = true;    // 256 x 512 tiles: a short last wave as half-width tiles
  std::mutex staging_mu;   // serialises b200gemm_bf16_nt_host calls on one handle
  std::vector<ScheduleEntry> schedules;
};

extern "C" int b200gemm_version(void) { return kVersion; }

extern "C" const char* b200gemm_strerror(int code) {
  switch (code) {
    case B200GEMM_OK: return "ok";
    case B200GEMM_ERR_INVALID_ARG: return "invalid argument (null handle or pointer, negative size)";
    case B200GEMM_ERR_UNSUPPORTED:
      return "unsupported layout (needs K % 8 == 0, ldc % 8 == 0, ldc >= N, 16-byte aligned pointers)";
    case B200GEMM_ERR_CUDA: return "a CUDA runtime or driver call failed";
    case B200GEMM_ERR_DEVICE_TIMEOUT: return "a bounded wait inside a kernel ran out of time";
    case B200GEMM_ERR_NO_DEVICE: return "no such CUDA device, or the device is not sm_100";
    case B200GEMM_ERR_TOO_LARGE: return "a dimension exceeds the supported range";
    default: return "unknown status code";
  }
}

extern "C" int b200gemm_create(b200gemm_t* out, int device) {
  if (out == nullptr) return B200GEMM_ERR_INVALID_ARG;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return B200GEMM_ERR_NO_DEVICE;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return B200GEMM_ERR_CUDA;
  if (prop.major != 10 || prop.minor != 0) return B200GEMM_ERR_NO_DEVICE;
  DeviceGuard guard(device);
  if (!guard.ok()) return B200GEMM_ERR_CUDA;
  if (tensor_map_encoder() == nullptr) return B200GEMM_ERR_CUDA;
  const int sms = prop.multiProcessorCount;
  const int cw[kNumWidths] = {prepare_kernel<CfgN256>(sms), prepare_kernel<CfgN512>(sms),
                              prepare_kernel<CfgN448>(sms), prepare_kernel<CfgN224>(sms),
                              prepare_kernel<CfgN192>(sms), prepare_kernel<CfgN128>(sms)};
  const int ce[kNumWidths] = {prepare_kernel<CfgE256>(sms), prepare_kernel<CfgE512>(sms),
                              prepare_kernel<CfgE448>(sms), prepare_kernel<CfgE224>(sms),
                              prepare_kernel<CfgE192>(sms), prepare_kernel<CfgE128>(sms)};
  for (int i = 0; i < kNumWidths; ++i)
    if (cw[i] <= 0 || ce[i] <= 0) return B200GEMM_ERR_CUDA;
  if (prepare_kernel<CfgN512H>(sms) <= 0 || prepare_kernel<CfgN448H>(sms) <= 0) return B200GEMM_ERR_CUDA;
  const int dc1 = prepare_decode_kernel<DecodeCfg<1>>(sms), dc2 = prepare_decode_kernel<DecodeCfg<2>>(sms),
            dc4 = prepare_decode_kernel<DecodeCfg<4>>(sms);
  if (dc1 <= 0 || dc2 <= 0 || dc4 <= 0) return B200GEMM_ERR_CUDA;
  const int dw1 = prepare_decode_kernel<DecodeCfg<1, 256>>(sms), dw2 = prepare_decode_kernel<DecodeCfg<2, 256>>(sms),
            dw3 = prepare_decode_kernel<DecodeCfg<3, 256>>(sms), dw4 = prepare_decode_kernel<DecodeCfg<4, 256>>(sms);
  if (dw1 <= 0 || dw2 <= 0 || dw3 <= 0 || dw4 <= 0) return B200GEMM_ERR_CUDA;
  const int sc2 = prepare_smallm1_kernel<SmallMCfg<2>>(sms), sc4 = prepare_smallm1_kernel<SmallMCfg<4>>(sms);
  if (sc2 <= 0 || sc4 <= 0) return B200GEMM_ERR_CUDA;

  auto* h = new b200gemm_handle();
  h->device = device;
  h->sm_count = prop.multiProcessorCount;
  h->decode_clusters[1] = dc1;
  h->decode_clusters[2] = dc2;
  h->decode_clusters[4] = dc4;
  h->decode256_clusters[1] = dw1;
  h->decode256_clusters[2] = dw2;
  h->decode256_clusters[3] = dw3;
  h->decode256_clusters[4] = dw4;
  h->smallm1_clusters[2] = sc2;
  h->smallm1_clusters[4] = sc4;
  h->max_clusters = cw[0];
  for (int i = 0; i < kNumWidths; ++i) {
    h->clusters_w[i] = cw[i];
    h->clusters_epi[i] = ce[i];
    if (cw[i] < h->max_clusters) h->max_clusters = cw[i];
  }
  if (cudaMalloc(&h->status_dev, 4 * sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(h->status_dev, 0, 4 * sizeof(unsigned int)) != cudaSuccess ||
      cudaMalloc(&h->tail_counters, kMaxTailCounters * sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(h->tail_counters, 0, kMaxTailCounters * sizeof(unsigned int)) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->tail_event, cudaEventDisableTiming) != cudaSuccess) {
    cudaFree(h->status_dev);
    cudaFree(h->tail_counters);
    delete h;
    return B200GEMM_ERR_CUDA;
  }
  *out = h;
  return B200GEMM_OK;
}

extern "C" void b200gemm_destroy(b200gemm_t h) {
  if (h == nullptr) return;
  {
    DeviceGuard guard(h->device);
    cudaDeviceSynchronize();
    for (auto& s : h->schedules) cudaFree(s.dev);
    cudaFree(h->status_dev);
    cudaFree(h->tail_ws);
    cudaFree(h->tail_counters);
    if (h->tail_event != nullptr) cudaEventDestroy(h->tail_event);
    HostStaging& st = h->staging;
    for (auto& b : st.set) {
      cudaFree(b.dA);
      cudaFree(b.dB);
      cudaFree(b.dC);
      if (b.ev_read != nullptr) cudaEventDestroy(b.ev_read);
      if (b.ev_done != nullptr) cudaEventDestroy(b.ev_done);
    }
    if (st.ready) {
      cudaStreamDestroy(st.s_h2d);
      cudaStreamDestroy(st.s_mma);
      cudaStreamDestroy(st.s_d2h);
      cudaEventDestroy(st.ev_start);
      cudaEventDestroy(st.ev_b);
      for (int i = 0; i < HostStaging::kMaxChunks; ++i) {
        cudaEventDestroy(st.ev_a[i]);
        cudaEventDestroy(st.ev_c[i]);
      }
    }
  }
  delete h;
}

extern "C" int b200gemm_set_timeout_ns(b200gemm_t h, unsigned long long timeout_ns) {
  if (h == nullptr) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->timeout_ns = timeout_ns;
  return B200GEMM_OK;
}

namespace {

// Tile schedule for a (tiles_m x tiles_n) grid, built on the device the
// first time the grid is seen and cached in the handle.  Caller holds h->mu.
int schedule_for(b200gemm_t h, uint32_t tiles_m, uint32_t tiles_n, cudaStream_t stream,
                 const uint32_t** out) {
  for (auto& s : h->schedules) {
    if (s.tiles_m == tiles_m && s.tiles_n == tiles_n && s.order == h->order && s.band == h->band) {
      s.last_use = ++h->tick;
      *out = s.dev;
      return B200GEMM_OK;
    }
  }
  if (h->schedules.size() >= kScheduleCacheSize) {
    size_t victim = 0;
    for (size_t i = 1; i < h->schedules.size(); ++i)
      if (h->schedules[i].last_use < h->schedules[victim].last_use) victim = i;
    cudaFree(h->schedules[victim].dev);  // synchronises the device
    h->schedules.erase(h->schedules.begin() + static_cast<long>(victim));
  }
  ScheduleEntry e;
  e.tiles_m = tiles_m;
  e.tiles_n = tiles_n;
  e.order = h->order;
  e.band = h->band;
  const size_t bytes = static_cast<size_t>(tiles_m) * tiles_n * sizeof(uint32_t);
  if (cudaMalloc(&e.dev, bytes) != cudaSuccess) return B200GEMM_ERR_CUDA;
  build_schedule_kernel<<<1, 1024, 0, stream>>>(tiles_m, tiles_n, e.order, e.band, e.dev);
  // Wait once so the table is valid for launches on any stream.
  if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(stream) != cudaSuccess) {
    cudaFree(e.dev);
    return B200GEMM_ERR_CUDA;
  }
  e.last_use = ++h->tick;
  h->schedules.push_back(e);
  *out = e.dev;
  return B200GEMM_OK;
}

// Tensor maps for one argument tuple, cached in the handle.  Caller holds h->mu.
int maps_for(b200gemm_t h, int M, int N, int K, const void* A, const void* B, void* C, int ldc,
             int b_rows, int c_type, CUtensorMap* ma, CUtensorMap* mb, CUtensorMap* mc) {
  MapEntry* slot = nullptr;
  for (auto& m : h->maps) {
    if (m.valid && m.a == A && m.b == B && m.c == C && m.M == M && m.N == N && m.K == K &&
        m.ldc == ldc && m.b_rows == b_rows && m.c_type == c_type) {
      slot = &m;
      break;
    }
  }
  if (slot == nullptr) {
    slot = &h->maps[0];
    for (auto& m : h->maps) {
      if (!m.valid) {
        slot = &m;
        break;
      }
      if (m.last_use < slot->last_use) slot = &m;
    }
    slot->valid = false;
    const uint64_t k = static_cast<uint64_t>(K);
    // A: 64 x 128 boxes, B: 64 x b_rows boxes (one 128-byte K row per operand
    // row), 128-byte swizzle as the MMA descriptors expect; C: 32 rows of 64
    // bytes (32 bf16 or 16 fp32 columns), 64-byte swizzle.  (e4m3 C is
    // written with plain stores; its map is encoded but unused.)
    const bool c_f32 = c_type == B200GEMM_OUT_F32, c_u8 = c_type == B200GEMM_OUT_E4M3;
    const uint64_t c_esize = c_f32 ? 4 : (c_u8 ? 1 : 2);
    if (!encode_2d(&slot->map_a, A, k, static_cast<uint64_t>(M), k * 2, kBlockK, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&slot->map_b, B, k, static_cast<uint64_t>(N), k * 2, kBlockK,
                   static_cast<uint32_t>(b_rows), CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&slot->map_c, C, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                   static_cast<uint64_t>(ldc) * c_esize, static_cast<uint32_t>(64 / c_esize),
                   kCBoxRows, CU_TENSOR_MAP_SWIZZLE_64B,
                   c_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                         : (c_u8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))) {
      return B200GEMM_ERR_CUDA;
    }
    slot->a = A;
    slot->b = B;
    slot->c = C;
    slot->M = M;
    slot->N = N;
    slot->K = K;
    slot->ldc = ldc;
    slot->b_rows = b_rows;
    slot->c_type = c_type;
    slot->valid = true;
  }
  slot->last_use = ++h->tick;
  *ma = slot->map_a;
  *mb = slot->map_b;
  *mc = slot->map_c;
  return B200GEMM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace {

bool tail_split_enabled_for(const b200gemm_handle* h) { return h->tail_split_enabled; }

// Tiles of the last wave that run as 256-column halves (0 = none): with T
// 256 x 512 tiles on G clusters, the R = T mod G tiles of the last wave when
// 2R <= G (a single partial wave counts: R = T < G).
int tail_half_for(const b200gemm_handle* h, int tiles, int clusters) {
  if (!h->tail_half_enabled || clusters <= 0) return 0;
  const int rem = tiles % clusters;
  return (rem > 0 && 2 * rem <= clusters) ? rem : 0;
}

// Instances that carry the K-split tail (GemmCfg::kTailSplit): the plain
// ones with one MMA column block (not the shared-A 512- and 448-wide ones).
bool tail_split_width(int width, bool fused) {
  return !fused && (width == 512 ? CfgN512::kTailSplit : (width == 448 ? CfgN448::kTailSplit : true));
}

// Tile width (one of kWidths) a call on this handle will use: the cheapest
// by tile_plan_cost (with the fused epilogue's cost when `epi` is given), the
// earlier entry of kWidths on a tie.
int choose_tile_width(const b200gemm_handle* h, int M, int N, int K,
                      const b200gemm_epilogue* epi = nullptr) {
  if (h->tile_width != 0) return h->tile_width;
  const uint32_t tiles_m = static_cast<uint32_t>((M + kTileM - 1) / kTileM);
  const int num_kb = (K + kBlockK - 1) / kBlockK;
  const int* clusters = epi != nullptr ? h->clusters_epi : h->clusters_w;
  int best = kWidths[0];
  double best_cost = tile_plan_cost(best, tiles_m, N, num_kb, clusters[0], epilogue_cost(epi, best));
  for (int i = 1; i < kNumWidths; ++i) {
    const double c = tile_plan_cost(kWidths[i], tiles_m, N, num_kb, clusters[i],
                                    epilogue_cost(epi, kWidths[i]));
    if (c < best_cost) {
      best_cost = c;
      best = kWidths[i];
    }
  }
  // Shared-A tiles with a half-width last wave replace the choice only when
  // clearly cheaper (3%): the model's margin of error is about that.
  if (h->tail_half_enabled && epi == nullptr) {
    const int base = best;
    double best_half = 0.97 * best_cost;
    for (int w : {512, 448}) {
      if (w == base) continue;
      const double c = tile_plan_cost(w, tiles_m, N, num_kb, clusters[width_index(w)], 0.0, true);
      if (c < best_half) {
        best_half = c;
        best = w;
      }
    }
  }
  return best;
}

// B rows of one CTA's tensor-map box for a tile width.
int b_box_rows(int width) { return width > 256 ? width / 4 : width / 2; }

cudaError_t launch_width(int width, bool fused, int clusters, cudaStream_t stream,
                         const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                         const GemmParams& p) {
  if (fused) {
    switch (width) {
      case 512: return launch_gemm<CfgE512>(clusters, stream, ma, mb, mc, p);
      case 448: return launch_gemm<CfgE448>(clusters, stream, ma, mb, mc, p);
      case 224: return launch_gemm<CfgE224>(clusters, stream, ma, mb, mc, p);
      case 192: return launch_gemm<CfgE192>(clusters, stream, ma, mb, mc, p);
      case 128: return launch_gemm<CfgE128>(clusters, stream, ma, mb, mc, p);
      default: return launch_gemm<CfgE256>(clusters, stream, ma, mb, mc, p);
    }
  }
  switch (width) {
    case 512:
      return p.tail_half ? launch_gemm<CfgN512H>(clusters, stream, ma, mb, mc, p)
                         : launch_gemm<CfgN512>(clusters, stream, ma, mb, mc, p);
    case 448:
      return p.tail_half ? launch_gemm<CfgN448H>(clusters, stream, ma, mb, mc, p)
                         : launch_gemm<CfgN448>(clusters, stream, ma, mb, mc, p);
    case 224: return launch_gemm<CfgN224>(clusters, stream, ma, mb, mc, p);
    case 192: return launch_gemm<CfgN192>(clusters, stream, ma, mb, mc, p);
    case 128: return launch_gemm<CfgN128>(clusters, stream, ma, mb, mc, p);
    default: return launch_gemm<CfgN256>(clusters, stream, ma, mb, mc, p);
  }
}

}  // namespace

namespace {

// K split for the small-M kernel, or 0 when the tiled kernel should run:
// M <= 256, N % 8 == 0 (its C stores are whole 16-byte groups), and the
// largest S in {4, 3, 2} ({4, 2} for M <= 128, whose 128 rows of A do not
// cut into three 32-row-aligned slices) whose N / 256 clusters of 2S CTAs are
// all co-resident (decode_clusters[S] for M <= 128, decode256_clusters[S]
// above, from the occupancy query: a cluster must fit in one GPC, so fewer
// than sm_count / 2S fit, and a second wave would double the time) while
// every CTA pair keeps at least two K blocks, else 1.  A split of 3 covers
// N = 4096 at 129..256 rows, where 16 clusters of 8 CTAs do not fit.
int decode_split(const b200gemm_handle* h, int M, int N, int K) {
  if (M > 256 || (N % 8) != 0 || K < 2 * kBlockK) return 0;
  const int clusters = (N + 255) / 256;
  const int num_kb = (K + kBlockK - 1) / kBlockK;
  const int* fit = M > 128 ? h->decode256_clusters : h->decode_clusters;
  for (int s : {4, 3, 2}) {
    if (s == 3 && (M <= 128 || !B200GEMM_SMALLM_SPLIT3)) continue;
    if (clusters <= fit[s] && num_kb >= 2 * s) return s;
  }
  return 1;
}

// Rows of C per CTA pair of the pair kernel (the map box height of C and of
// the residual): DecodeCfg<S, NT>::kSliceRows.
uint32_t decode_slice_rows(int nt, int split) {
  return static_cast<uint32_t>((nt / split + 31) / 32 * 32);
}

// Which small-M kernel a shape takes: kind 0 = none (tiled kernel), 2 = the
// pair kernel (256 rows of B per CTA pair), 3 = the single-CTA kernel (128
// rows of B per CTA); split = its K split.  The pair kernel keeps more of B
// in flight per SM (16 of its 24 KB stages against 16 of 32), so the
// single-CTA kernel is taken only where it puts at least 1.5x the CTAs to
// work, i.e. where the pair kernel's clusters cannot all co-reside at a
// useful split (narrow N: N = 4096 gets 128 CTAs instead of 64).
struct SmallMPlan {
  int kind;
  int split;
  int nt = 0;        // pair kernel: rows of A per MMA (128 or 256)
  int clusters = 0;  // clusters launched
};

// Device-side epilogue arguments of a call (identity when epi is null).
EpiArgs epi_args(const b200gemm_epilogue* epi) {
  EpiArgs e{};
  e.flags = 0;
  e.act = B200GEMM_ACT_NONE;
  e.out_type = B200GEMM_OUT_BF16;
  e.alpha = 1.0f;
  e.beta = 0.0f;
  e.out_scale = 1.0f;
  if (epi != nullptr) {
    e.flags = (epi->bias != nullptr ? kEpiBias : 0u) | (epi->residual != nullptr ? kEpiResidual : 0u);
    e.act = epi->activation;
    e.out_type = epi->out_type;
    e.alpha = epi->alpha;
    e.beta = epi->beta;
    e.out_scale = epi->out_scale == 0.0f ? 1.0f : epi->out_scale;
    e.bias = static_cast<const uint16_t*>(epi->bias);
    e.residual = static_cast<const uint16_t*>(epi->residual);
    e.ldr = epi->ldr;
  }
  return e;
}

// C of the small-M kernels: boxes of 32 columns x slice_rows rows in the
// output type, no swizzle (the transposing staging buffer is row-major).
// The residual of a fused epilogue for the small-M kernels: the same boxes
// (32 columns x slice_rows rows) of the bf16 M x N matrix with pitch ldr;
// without a residual the C map stands in (the kernels then never read it).
bool encode_smallm_r(CUtensorMap* mr, const CUtensorMap& mc, const b200gemm_epilogue* epi, int M, int N,
                     uint32_t slice_rows) {
  if (epi == nullptr || epi->residual == nullptr) {
    *mr = mc;
    return true;
  }
  return encode_2d(mr, epi->residual, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                   static_cast<uint64_t>(epi->ldr) * 2, 32, slice_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool encode_smallm_c(CUtensorMap* mc, void* C, int M, int N, int ldc, uint32_t slice_rows, int out_type) {
  const bool f32 = out_type == B200GEMM_OUT_F32, u8 = out_type == B200GEMM_OUT_E4M3;
  const uint64_t esize = f32 ? 4 : (u8 ? 1 : 2);
  return encode_2d(mc, C, static_cast<uint64_t>(N), static_cast<uint64_t>(M), static_cast<uint64_t>(ldc) * esize,
                   32, slice_rows, CU_TENSOR_MAP_SWIZZLE_NONE,
                   f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                       : (u8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16));
}

// 257..B200GEMM_SMALLM_MAX_ROWS rows of A: the pair kernel over blocks of
// 128 or 256 rows of A (clusters = N / 256 x M / block, K split over 2 or 4
// pairs, so every slice is whole 32-row chunks inside its block).  All its
// clusters must fit at once.  Measured on B200, both kernels are then bound
// by how fast each CTA is fed from L2 (~12-15 ns per KB); so the first
// layout that fits -- 128-row blocks before 256-row ones (their smaller
// partial sums cost less to exchange), split 4 where every pair gets at
// least 4 K blocks -- is taken where a CTA's bytes (operand K blocks plus
// the partial sums it exchanges) are at most 0.8 of what a CTA of the tiled
// kernel loads (waves x K blocks x (16 + width / 16) KB).  {0, 0} otherwise,
// and while a tile width is forced (that asks for the tiled kernel).  A fused
// epilogue does not change the choice: such a call runs the kernel the plain
// call runs.
SmallMPlan smallm_blocks_plan(const b200gemm_handle* h, int M, int N, int K) {
  if (h->tile_width != 0 || M <= 256 || M > B200GEMM_SMALLM_MAX_ROWS || (N % 8) != 0 || K < 2 * kBlockK) return {0, 0};
  const int num_kb = (K + kBlockK - 1) / kBlockK;
  const int n_blocks = (N + 255) / 256;
  SmallMPlan pick{0, 0};
  double pair_kb = 0.0;  // KB one CTA loads and exchanges
  for (int nt : {128, 256}) {
    const int clusters = n_blocks * ((M + nt - 1) / nt);
    const int* fit = nt == 256 ? h->decode256_clusters : h->decode_clusters;
    for (int s : {4, 2}) {
      if (clusters > fit[s] || num_kb < (s == 4 ? 16 : 4)) continue;
      pick = SmallMPlan{2, s};
      pick.nt = nt;
      pick.clusters = clusters;
      pair_kb = ((num_kb + s - 1) / s) * (16.0 + nt / 16.0) + nt / 2.0 * (s - 1) / s;
      break;
    }
    if (pick.kind != 0) break;
  }
  if (pick.kind == 0) return pick;
  const int width = choose_tile_width(h, M, N, K);
  const int maxc = h->clusters_w[width_index(width)];
  const int tiles = ((M + kTileM - 1) / kTileM) * ((N + width - 1) / width);
  const int waves = (tiles + maxc - 1) / maxc;
  const double tiled_kb = static_cast<double>(waves) * num_kb * (16.0 + width / 16.0);
  if (pair_kb > 0.8 * tiled_kb) return {0, 0};
  return pick;
}

SmallMPlan smallm_plan(const b200gemm_handle* h, int M, int N, int K) {
  if (M > 256) return smallm_blocks_plan(h, M, N, K);
  const int sp = decode_split(h, M, N, K);
  if (sp == 0) return {0, 0};
  SmallMPlan pair{2, sp};
  pair.nt = M > 128 ? 256 : 128;
  pair.clusters = (N + 255) / 256;
  if (M > 128) return pair;  // the single-CTA kernel covers at most 128 rows of A
  const int ctas_pair = (N + 255) / 256 * 2 * sp;
  const int clusters1 = (N + 127) / 128;
  const int num_kb = (K + kBlockK - 1) / kBlockK;
  for (int s : {4, 2}) {  // (without a K split it never has 1.5x the pair kernel's CTAs)
    if (clusters1 <= h->smallm1_clusters[s] && num_kb >= 2 * s) {
      const int ctas_single = clusters1 * s;
      if (2 * ctas_single >= 3 * ctas_pair && ctas_single <= h->sm_count) {
        SmallMPlan one{3, s};
        one.clusters = clusters1;
        return one;
      }
      break;
    }
  }
  return pair;
}

int run_smallm1(b200gemm_t h, int split, int M, int N, int K, const void* A, const void* B, void* C,
                int ldc, cudaStream_t stream, unsigned long long timeout_ns, int pdl,
                const b200gemm_epilogue* epi) {
  const uint64_t k = static_cast<uint64_t>(K);
  CUtensorMap ma, mb, mc, mr;
  const uint32_t slice_rows = static_cast<uint32_t>(128 / split);
  const EpiArgs ea = epi_args(epi);
  if (!encode_2d(&ma, A, k, static_cast<uint64_t>(M), k * 2, kBlockK, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&mb, B, k, static_cast<uint64_t>(N), k * 2, kBlockK, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_smallm_c(&mc, C, M, N, ldc, slice_rows, ea.out_type) ||
      !encode_smallm_r(&mr, mc, epi, M, N, slice_rows)) {
    return B200GEMM_ERR_CUDA;
  }
  SmallMParams p{};
  p.epi = ea;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_kb = (K + kBlockK - 1) / kBlockK;
  p.kb_per_split = (p.num_kb + split - 1) / split;
  p.status = h->status_dev;
  p.timeout_ns = timeout_ns;
  p.pdl = pdl;
  cudaError_t e;
  if (split == 4) e = launch_smallm1<SmallMCfg<4>>(stream, ma, mb, mc, mr, p);
  else if (split == 2) e = launch_smallm1<SmallMCfg<2>>(stream, ma, mb, mc, mr, p);
  else return B200GEMM_ERR_INVALID_ARG;  // smallm_plan picks split 2 or 4
  return e == cudaSuccess ? B200GEMM_OK : B200GEMM_ERR_CUDA;
}

int run_decode(b200gemm_t h, int split, int nt, int M, int N, int K, const void* A, const void* B,
               void* C, int ldc, cudaStream_t stream, unsigned long long timeout_ns, int pdl,
               const b200gemm_epilogue* epi) {
  const uint64_t k = static_cast<uint64_t>(K);
  CUtensorMap ma, mb, mc, mr;  // nt: rows of A one MMA covers (one M block)
  const uint32_t slice_rows = decode_slice_rows(nt, split);
  const EpiArgs ea = epi_args(epi);
  if (!encode_2d(&ma, A, k, static_cast<uint64_t>(M), k * 2, kBlockK, nt / 2, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&mb, B, k, static_cast<uint64_t>(N), k * 2, kBlockK, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_smallm_c(&mc, C, M, N, ldc, slice_rows, ea.out_type) ||
      !encode_smallm_r(&mr, mc, epi, M, N, slice_rows)) {
    return B200GEMM_ERR_CUDA;
  }
  DecodeParams p{};
  p.epi = ea;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_kb = (K + kBlockK - 1) / kBlockK;
  p.kb_per_split = (p.num_kb + split - 1) / split;
  const int kps = nt == 256 ? DecodeCfg<1, 256>::kKps : DecodeCfg<1, 128>::kKps;
  p.kb_per_split = (p.kb_per_split + kps - 1) / kps * kps;  // whole stages per pair
  p.status = h->status_dev;
  p.timeout_ns = timeout_ns;
  p.pdl = pdl;
  p.n_blocks = (N + 255) / 256;
  cudaError_t e;
  if (nt == 256) {
    if (split == 4) e = launch_decode<DecodeCfg<4, 256>>(stream, ma, mb, mc, mr, p);
    else if (split == 3) e = launch_decode<DecodeCfg<3, 256>>(stream, ma, mb, mc, mr, p);
    else if (split == 2) e = launch_decode<DecodeCfg<2, 256>>(stream, ma, mb, mc, mr, p);
    else e = launch_decode<DecodeCfg<1, 256>>(stream, ma, mb, mc, mr, p);
  } else {
    if (split == 4) e = launch_decode<DecodeCfg<4>>(stream, ma, mb, mc, mr, p);
    else if (split == 2) e = launch_decode<DecodeCfg<2>>(stream, ma, mb, mc, mr, p);
    else e = launch_decode<DecodeCfg<1>>(stream, ma, mb, mc, mr, p);
  }
  return e == cudaSuccess ? B200GEMM_OK : B200GEMM_ERR_CUDA;
}

}  // namespace

extern "C" int b200gemm_small_m_split(b200gemm_t h, int M, int N, int K) {
  if (h == nullptr || M <= 0 || N <= 0 || K < 0) return 0;
  std::lock_guard<std::mutex> lock(h->mu);
  return h->small_m != 0 ? smallm_plan(h, M, N, K).split : 0;
}

extern "C" int b200gemm_set_small_m(b200gemm_t h, int mode) {
  if (h == nullptr || mode < -1 || mode > 1) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->small_m = mode;
  return B200GEMM_OK;
}

static_assert(B200GEMM_PDL_OFF == kPdlOff && B200GEMM_PDL_ON == kPdlOn &&
                  B200GEMM_PDL_WEIGHTS_EARLY == kPdlWeightsEarly,
              "header and kernel agree on the launch-overlap modes");

extern "C" int b200gemm_set_pdl(b200gemm_t h, int mode) {
  if (h == nullptr || mode < B200GEMM_PDL_OFF || mode > B200GEMM_PDL_WEIGHTS_EARLY) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->pdl = mode;
  return B200GEMM_OK;
}

namespace {
int gemm_device(b200gemm_t h, int M, int N, int K, const void* A, const void* B, void* C, int ldc,
                void* stream_ptr, bool allow_small_m, int npeers = 0,
                void* const* peers = nullptr, const b200gemm_epilogue* epi = nullptr, void* mc_c = nullptr);
}  // namespace

extern "C" int b200gemm_bf16_nt(b200gemm_t h, int M, int N, int K, const void* A, const void* B,
                                void* C, int ldc, void* stream_ptr) {
  return gemm_device(h, M, N, K, A, B, C, ldc, stream_ptr, true);
}

extern "C" int b200gemm_bf16_nt_epilogue(b200gemm_t h, int M, int N, int K, const void* A,
                                         const void* B, void* C, int ldc,
                                         const b200gemm_epilogue* epi, void* stream_ptr) {
  return gemm_device(h, M, N, K, A, B, C, ldc, stream_ptr, /*allow_small_m=*/true, 0, nullptr, epi);
}

extern "C" int b200gemm_bf16_nt_allgather(b200gemm_t h, int M, int N, int K, const void* A,
                                          const void* B, void* C, int ldc, void* const* peer_C,
                                          int npeers, void* stream_ptr) {
  if (npeers < 0 || npeers > GemmParams::kMaxPeers || (npeers > 0 && peer_C == nullptr))
    return B200GEMM_ERR_INVALID_ARG;
  for (int i = 0; i < npeers; ++i) {
    if (peer_C[i] == nullptr) return B200GEMM_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(peer_C[i]) & 15u) != 0) return B200GEMM_ERR_UNSUPPORTED;
  }
  if ((N % 8) != 0) return B200GEMM_ERR_UNSUPPORTED;  // peer rows are copied in 16-byte pieces
  if (K == 0 && M > 0 && N > 0) return B200GEMM_ERR_UNSUPPORTED;  // the peers' blocks would stay unwritten
  return gemm_device(h, M, N, K, A, B, C, ldc, stream_ptr, /*allow_small_m=*/false, npeers, peer_C);
}

extern "C" int b200gemm_bf16_nt_allgather_multicast(b200gemm_t h, int M, int N, int K, const void* A,
                                                    const void* B, void* C, int ldc, void* mc_C,
                                                    void* stream_ptr) {
  if (mc_C == nullptr) return B200GEMM_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(mc_C) & 15u) != 0 || (N % 8) != 0) return B200GEMM_ERR_UNSUPPORTED;
  if (K == 0 && M > 0 && N > 0) return B200GEMM_ERR_UNSUPPORTED;  // every rank's block would stay unwritten
  return gemm_device(h, M, N, K, A, B, C, ldc, stream_ptr, /*allow_small_m=*/false, 0, nullptr, nullptr,
                     mc_C);
}

extern "C" int b200gemm_ipc_get_handle(const void* dev_ptr, void* handle_out,
                                       unsigned long long* offset_out) {
  if (dev_ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return B200GEMM_ERR_INVALID_ARG;
  // A handle names the whole allocation, so report where dev_ptr sits in it
  // (a caching allocator may hand out pointers inside larger blocks).
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
    }
  });
  if (range_fn == nullptr) return B200GEMM_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return B200GEMM_ERR_CUDA;
  cudaIpcMemHandle_t hnd;
  if (cudaIpcGetMemHandle(&hnd, reinterpret_cast<void*>(base)) != cudaSuccess) return B200GEMM_ERR_CUDA;
  static_assert(sizeof(hnd) <= B200GEMM_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &hnd, sizeof(hnd));
  *offset_out = static_cast<unsigned long long>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return B200GEMM_OK;
}

extern "C" int b200gemm_ipc_open(const void* handle, void** dev_ptr_out) {
  if (handle == nullptr || dev_ptr_out == nullptr) return B200GEMM_ERR_INVALID_ARG;
  cudaIpcMemHandle_t hnd;
  std::memcpy(&hnd, handle, sizeof(hnd));
  if (cudaIpcOpenMemHandle(dev_ptr_out, hnd, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return B200GEMM_ERR_CUDA;
  return B200GEMM_OK;
}

extern "C" int b200gemm_ipc_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return B200GEMM_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? B200GEMM_OK : B200GEMM_ERR_CUDA;
}

namespace {

// The device-pointer GEMM.  `allow_small_m` = false keeps a call on the
// tiled kernel (used for the row chunks of a larger host-staged problem, so
// chunking never changes which kernel, and hence which summation order, an
// element gets).
int gemm_device(b200gemm_t h, int M, int N, int K, const void* A, const void* B, void* C, int ldc,
                void* stream_ptr, bool allow_small_m, int npeers, void* const* peers,
                const b200gemm_epilogue* epi, void* mc_c) {
  if (h == nullptr || M < 0 || N < 0 || K < 0) return B200GEMM_ERR_INVALID_ARG;
  const bool fused = epi != nullptr;
  const int c_type = fused ? epi->out_type : B200GEMM_OUT_BF16;
  if (fused) {
    if (c_type != B200GEMM_OUT_BF16 && c_type != B200GEMM_OUT_F32 && c_type != B200GEMM_OUT_E4M3)
      return B200GEMM_ERR_INVALID_ARG;
    if (epi->activation < B200GEMM_ACT_NONE || epi->activation > B200GEMM_ACT_SILU)
      return B200GEMM_ERR_INVALID_ARG;
    if (epi->residual != nullptr && (epi->ldr < N || (epi->ldr % 8) != 0 || !aligned16(epi->residual)))
      return B200GEMM_ERR_UNSUPPORTED;
    if (epi->bias != nullptr && !aligned16(epi->bias)) return B200GEMM_ERR_UNSUPPORTED;
  }
  if (M == 0 || N == 0) return B200GEMM_OK;
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr))) return B200GEMM_ERR_INVALID_ARG;
  // C rows start on 16-byte boundaries: ldc a multiple of 16 bytes.
  const int ldc_group = c_type == B200GEMM_OUT_F32 ? 4 : (c_type == B200GEMM_OUT_E4M3 ? 16 : 8);
  if (ldc < N || (ldc % ldc_group) != 0 || (K % 8) != 0) return B200GEMM_ERR_UNSUPPORTED;
  if (fused && K == 0) return B200GEMM_ERR_UNSUPPORTED;  // the kernel needs one K block
  if (!aligned16(C) || (K > 0 && (!aligned16(A) || !aligned16(B)))) return B200GEMM_ERR_UNSUPPORTED;
  const uint32_t tiles_m = static_cast<uint32_t>((M + kTileM - 1) / kTileM);
  // Tile coordinates are 16-bit: bound the grid of the narrowest width.
  if (tiles_m > 0xFFFFu || static_cast<uint32_t>((N + 127) / 128) > 0xFFFFu)
    return B200GEMM_ERR_TOO_LARGE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  DeviceGuard guard(h->device);
  if (!guard.ok()) return B200GEMM_ERR_CUDA;

  if (K == 0) {  // empty sum: C = 0
    return cudaMemset2DAsync(C, static_cast<size_t>(ldc) * 2, 0, static_cast<size_t>(N) * 2,
                             static_cast<size_t>(M), stream) == cudaSuccess
               ? B200GEMM_OK
               : B200GEMM_ERR_CUDA;
  }

  // Small M: stream B with every SM (operands swapped, K split in-cluster).
  SmallMPlan sm{0, 0};
  unsigned long long decode_timeout;
  int pdl;
  // Their C stores clip N in 16-byte units: e4m3 output needs N % 16 == 0.
  const bool smallm_ok = allow_small_m && npeers == 0 && mc_c == nullptr &&
                         (c_type != B200GEMM_OUT_E4M3 || (N % 16) == 0);
  {
    std::lock_guard<std::mutex> lock(h->mu);
    if (smallm_ok && h->small_m != 0) sm = smallm_plan(h, M, N, K);
    decode_timeout = h->timeout_ns;
    pdl = h->pdl;
  }
  if (sm.kind == 2) return run_decode(h, sm.split, sm.nt, M, N, K, A, B, C, ldc, stream, decode_timeout, pdl, epi);
  if (sm.kind == 3) return run_smallm1(h, sm.split, M, N, K, A, B, C, ldc, stream, decode_timeout, pdl, epi);

  CUtensorMap ma, mb, mc;
  const uint32_t* sched = nullptr;
  unsigned long long timeout_ns;
  int width;
  uint32_t tiles_n;
  {
    std::lock_guard<std::mutex> lock(h->mu);
    width = choose_tile_width(h, M, N, K, epi);
    tiles_n = static_cast<uint32_t>((N + width - 1) / width);
    int rc = schedule_for(h, tiles_m, tiles_n, stream, &sched);
    if (rc != B200GEMM_OK) return rc;
    rc = maps_for(h, M, N, K, A, B, C, ldc, b_box_rows(width), c_type, &ma, &mb, &mc);
    if (rc != B200GEMM_OK) return rc;
    timeout_ns = h->timeout_ns;
  }

  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_kb = (K + kBlockK - 1) / kBlockK;
  p.num_tiles = static_cast<int>(tiles_m * tiles_n);
  p.tiles = sched;
  p.status = h->status_dev;
  p.timeout_ns = timeout_ns;
  p.C = static_cast<uint16_t*>(C);
  p.ldc = ldc;
  p.npeers = npeers;
  for (int i = 0; i < GemmParams::kMaxPeers; ++i)
    p.peer_c[i] = i < npeers ? static_cast<uint8_t*>(peers[i]) : nullptr;
  p.mc_c = static_cast<uint8_t*>(mc_c);
  // Launch overlap (no B-first variant here: the tile table comes first);
  // the all-gather forms keep plain stream order.
  p.pdl = (pdl != kPdlOff && npeers == 0 && mc_c == nullptr) ? kPdlOn : kPdlOff;

  p.epi_flags = 0;
  p.act = B200GEMM_ACT_NONE;
  p.out_type = c_type;
  p.alpha = 1.0f;
  p.beta = 0.0f;
  p.out_scale = 1.0f;
  p.bias = nullptr;
  p.residual = nullptr;
  p.ldr = 0;
  if (fused) {
    p.epi_flags = (epi->bias != nullptr ? kEpiBias : 0u) | (epi->residual != nullptr ? kEpiResidual : 0u);
    p.act = epi->activation;
    p.alpha = epi->alpha;
    p.beta = epi->beta;
    p.bias = static_cast<const uint16_t*>(epi->bias);
    p.residual = static_cast<const uint16_t*>(epi->residual);
    p.ldr = epi->ldr;
    p.out_scale = epi->out_scale == 0.0f ? 1.0f : epi->out_scale;
  }

  const int max_clusters = fused ? h->clusters_epi[width_index(width)] : h->clusters_w[width_index(width)];
  int clusters = p.num_tiles < max_clusters ? p.num_tiles : max_clusters;
  // Split the last partial wave along K when it leaves clusters idle (plain
  // epilogue only: the split tiles' reduction writes bf16 directly).  With
  // fewer tiles than clusters the one wave is all tail: every tile is split.
  const int sk = (tail_split_enabled_for(h) && tail_split_width(width, fused))
                     ? tail_split_for(p.num_tiles, max_clusters, p.num_kb)
                     : 1;
  p.tail_start = p.num_tiles;
  p.tail_split = 1;
  p.tail_kb = p.num_kb;
  p.num_units = p.num_tiles;
  p.workspace = nullptr;
  p.tail_counters = nullptr;
  bool tail_on = false;
  if (sk >= 2) {
    const int rem = p.num_tiles % max_clusters;
    const size_t need = static_cast<size_t>(rem) * sk * 2 * 128 * width * sizeof(float);
    std::lock_guard<std::mutex> lock(h->mu);
    bool have_ws = h->tail_ws_bytes >= need;
    if (!have_ws && 2 * rem <= kMaxTailCounters) {
      cudaFree(h->tail_ws);  // waits for launches still using the old workspace
      h->tail_ws = nullptr;
      h->tail_ws_bytes = 0;
      if (cudaMalloc(&h->tail_ws, need) == cudaSuccess) {
        h->tail_ws_bytes = need;
        have_ws = true;
      }
    }
    if (have_ws && 2 * rem <= kMaxTailCounters) {
      p.tail_start = p.num_tiles - rem;
      p.tail_split = sk;
      p.tail_kb = (p.num_kb + sk - 1) / sk;
      p.num_units = p.tail_start + rem * sk;
      clusters = p.num_units < max_clusters ? p.num_units : max_clusters;
      p.workspace = h->tail_ws;
      p.tail_counters = h->tail_counters;
      tail_on = true;
      if (h->tail_event_recorded && cudaStreamWaitEvent(stream, h->tail_event, 0) != cudaSuccess)
        return B200GEMM_ERR_CUDA;
    }
  }

  // 256 x 512 tiles: a last wave of at most half as many tiles as clusters
  // runs as 256-column halves on twice the clusters (plain epilogue only).
  if (!tail_on && (width == 512 || width == 448) && !fused && tail_half_for(h, p.num_tiles, max_clusters) > 0) {
    const int rem = tail_half_for(h, p.num_tiles, max_clusters);
    p.tail_start = p.num_tiles - rem;
    p.tail_half = 1;
    p.num_units = p.tail_start + 2 * rem;
    clusters = p.num_units < max_clusters ? p.num_units : max_clusters;
  }

  // One wave of whole tiles: each cluster computes its tile from its index
  // instead of loading it from the table (a dependent global load before
  // the first operand load, which matters for small, latency-bound calls).
  if (p.num_units == p.num_tiles && p.num_tiles <= clusters) p.direct_tiles_n = static_cast<int>(tiles_n);
  const cudaError_t e = launch_width(width, fused, clusters, stream, ma, mb, mc, p);
  if (e == cudaSuccess && tail_on) {
    std::lock_guard<std::mutex> lock(h->mu);
    if (cudaEventRecord(h->tail_event, stream) != cudaSuccess) return B200GEMM_ERR_CUDA;
    h->tail_event_recorded = true;
  }
  return e == cudaSuccess ? B200GEMM_OK : B200GEMM_ERR_CUDA;
}

}  // namespace

extern "C" int b200gemm_plan(b200gemm_t h, int M, int N, int K, int* plan) {
  if (h == nullptr || plan == nullptr || M <= 0 || N <= 0 || K <= 0) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  for (int i = 0; i < 6; ++i) plan[i] = 0;
  const SmallMPlan sm = h->small_m != 0 ? smallm_plan(h, M, N, K) : SmallMPlan{0, 0};
  if (sm.kind != 0) {
    plan[0] = sm.kind;  // 2: small-M pair kernel, 3: small-M single-CTA kernel
    plan[1] = sm.kind == 2 ? 256 : 128;  // rows of B per cluster
    plan[2] = sm.clusters;
    plan[3] = sm.clusters;
    plan[5] = sm.split;
    return B200GEMM_OK;
  }
  const int width = choose_tile_width(h, M, N, K);
  const int tiles = ((M + kTileM - 1) / kTileM) * ((N + width - 1) / width);
  const int maxc = h->clusters_w[width_index(width)];
  const int num_kb = (K + kBlockK - 1) / kBlockK;
  const int sk = (h->tail_split_enabled && tail_split_width(width, false)) ? tail_split_for(tiles, maxc, num_kb) : 1;
  const int halves = (sk < 2 && (width == 512 || width == 448)) ? tail_half_for(h, tiles, maxc) : 0;
  const int units = tiles + (sk >= 2 ? (tiles % maxc) * (sk - 1) : 0) + halves;
  const int clusters = units < maxc ? units : maxc;
  plan[0] = 1;  // tiled kernel
  plan[1] = width;
  plan[2] = tiles;
  plan[3] = clusters;
  plan[4] = sk >= 2 ? sk : (halves > 0 ? -2 : 1);
  return B200GEMM_OK;
}

extern "C" int b200gemm_set_tail_half(b200gemm_t h, int enable) {
  if (h == nullptr) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->tail_half_enabled = enable != 0;
  return B200GEMM_OK;
}

extern "C" int b200gemm_set_tail_split(b200gemm_t h, int enable) {
  if (h == nullptr) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->tail_split_enabled = enable != 0;
  return B200GEMM_OK;
}

extern "C" int b200gemm_set_tile_width(b200gemm_t h, int width) {
  if (h == nullptr || (width != 0 && width_index(width) < 0)) return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->tile_width = width;
  return B200GEMM_OK;
}

extern "C" int b200gemm_tile_width_for(b200gemm_t h, int M, int N, int K) {
  if (h == nullptr || M <= 0 || N <= 0 || K < 0) return 0;
  std::lock_guard<std::mutex> lock(h->mu);
  return choose_tile_width(h, M, N, K);
}

extern "C" int b200gemm_last_device_status(b200gemm_t h, unsigned int* detail) {
  if (h == nullptr) return B200GEMM_ERR_INVALID_ARG;
  DeviceGuard guard(h->device);
  if (!guard.ok()) return B200GEMM_ERR_CUDA;
  unsigned int words[4] = {0, 0, 0, 0};
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(words, h->status_dev, sizeof(words), cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemset(h->status_dev, 0, sizeof(words)) != cudaSuccess) {
    return B200GEMM_ERR_CUDA;
  }
  if (detail != nullptr) std::memcpy(detail, words, sizeof(words));
  return words[0] == 0 ? B200GEMM_OK : static_cast<int>(words[0]);
}

extern "C" int b200gemm_selftest_watchdog(b200gemm_t h, unsigned long long timeout_ns,
                                          void* stream_ptr) {
  if (h == nullptr) return B200GEMM_ERR_INVALID_ARG;
  DeviceGuard guard(h->device);
  if (!guard.ok()) return B200GEMM_ERR_CUDA;
  watchdog_selftest_kernel<<<2, 32, 0, static_cast<cudaStream_t>(stream_ptr)>>>(h->status_dev,
                                                                               timeout_ns);
  return cudaGetLastError() == cudaSuccess ? B200GEMM_OK : B200GEMM_ERR_CUDA;
}

extern "C" int b200gemm_device_info(b200gemm_t h, int* sm_count, int* max_clusters) {
  if (h == nullptr) return B200GEMM_ERR_INVALID_ARG;
  if (sm_count != nullptr) *sm_count = h->sm_count;
  if (max_clusters != nullptr) *max_clusters = h->max_clusters;
  return B200GEMM_OK;
}

extern "C" int b200gemm_set_schedule(b200gemm_t h, int order, int band) {
  if (h == nullptr || (order != kOrderHilbert && order != kOrderBands) || band < 1 || band > 0xFFFF)
    return B200GEMM_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(h->mu);
  h->order = order;
  h->band = static_cast<uint32_t>(band);
  return B200GEMM_OK;
}

extern "C" int b200gemm_schedule_host(unsigned int tiles_m, unsigned int tiles_n, int order,
                                      int band, unsigned int* out) {
  if (out == nullptr || tiles_m == 0 || tiles_n == 0 || tiles_m > 0xFFFFu || tiles_n > 0xFFFFu ||
      (order != kOrderHilbert && order != kOrderBands) || band < 1 || band > 0xFFFF)
    return B200GEMM_ERR_INVALID_ARG;
  build_schedule_host(tiles_m, tiles_n, order, static_cast<uint32_t>(band), out);
  return B200GEMM_OK;
}

extern "C" int b200gemm_run_kernel(int M, int N, int K, const void* A, const void* B, void* C,
                                   int* DB) {
  (void)DB;
  static std::mutex mu;
  static b200gemm_t handles[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B200GEMM_ERR_NO_DEVICE;
  b200gemm_t h;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (handles[dev] == nullptr) {
      const int rc = b200gemm_create(&handles[dev], dev);
      if (rc != B200GEMM_OK) return rc;
    }
    h = handles[dev];
  }
  return b200gemm_bf16_nt(h, M, N, K, A, B, C, N, nullptr);
}

// ---------------------------------------------------------------------------
// Host-resident operands.  The problem is cut into row chunks of A and C;
// three streams overlap the host->device copies of A chunks, the GEMM of the
// previous chunk and the device->host copy of the chunk before it.  B is
// copied first because every chunk needs all of it.
namespace {

bool ensure_capacity(void** buf, size_t* cap, size_t bytes) {
  if (*cap >= bytes) return true;
  cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  if (cudaMalloc(buf, bytes) != cudaSuccess) return false;
  *cap = bytes;
  return true;
}

bool prepare_staging(HostStaging& st) {
  if (st.ready) return true;
  bool ok = cudaStreamCreateWithFlags(&st.s_h2d, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&st.s_mma, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&st.s_d2h, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&st.ev_start, cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&st.ev_b, cudaEventDisableTiming) == cudaSuccess;
  for (auto& b : st.set) {
    ok = ok && cudaEventCreateWithFlags(&b.ev_read, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&b.ev_done, cudaEventDisableTiming) == cudaSuccess;
  }
  for (int i = 0; ok && i < HostStaging::kMaxChunks; ++i) {
    ok = cudaEventCreateWithFlags(&st.ev_a[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&st.ev_c[i], cudaEventDisableTiming) == cudaSuccess;
  }
  st.ready = ok;
  return ok;
}

}  // namespace

extern "C" int b200gemm_bf16_nt_host(b200gemm_t h, int M, int N, int K, const void* hA,
                                     const void* hB, void* hC, int ldc, void* stream_ptr) {
  if (h == nullptr || M < 0 || N < 0 || K < 0) return B200GEMM_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return B200GEMM_OK;
  if (hC == nullptr || (K > 0 && (hA == nullptr || hB == nullptr))) return B200GEMM_ERR_INVALID_ARG;
  if (ldc < N || (K % 8) != 0) return B200GEMM_ERR_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  DeviceGuard guard(h->device);
  if (!guard.ok()) return B200GEMM_ERR_CUDA;
  std::lock_guard<std::mutex> lock(h->staging_mu);
  HostStaging& st = h->staging;
  const size_t ldc_dev = (static_cast<size_t>(N) + 7) & ~static_cast<size_t>(7);
  const size_t bytesA = static_cast<size_t>(M) * K * 2, bytesB = static_cast<size_t>(N) * K * 2;
  const size_t bytesC = static_cast<size_t>(M) * ldc_dev * 2;
  if (!prepare_staging(st)) return B200GEMM_ERR_CUDA;
  HostStaging::Buffers& buf = st.set[st.next];
  // A buffer about to be freed and grown may still be in use by the call
  // two back: wait for it first (the usual case, same size, never waits).
  if ((buf.capA < bytesA || buf.capB < bytesB || buf.capC < bytesC) &&
      cudaEventSynchronize(buf.ev_done) != cudaSuccess) {
    return B200GEMM_ERR_CUDA;
  }
  if (!ensure_capacity(&buf.dA, &buf.capA, bytesA > 0 ? bytesA : 16) ||
      !ensure_capacity(&buf.dB, &buf.capB, bytesB > 0 ? bytesB : 16) ||
      !ensure_capacity(&buf.dC, &buf.capC, bytesC)) {
    return B200GEMM_ERR_CUDA;
  }
  st.next ^= 1;
  // Shapes the small-M kernel takes (M <= 256, or a small shape it covers in
  // blocks of A's rows) run as one GEMM after one upload of A, so that the
  // result is the device path's bit for bit: the tiled kernel sums an
  // element's K products in the same order whatever rows a chunk holds, the
  // small-M kernel's K split does not.
  bool whole = M <= 256;
  if (!whole) {
    std::lock_guard<std::mutex> plan_lock(h->mu);
    whole = h->small_m != 0 && smallm_plan(h, M, N, K).kind != 0;
  }
  // Chunks: whole 256-row tiles, about 3 when M allows.  Calls back to back
  // (the next call's uploads overlap this one's GEMMs and copy-out) ran
  // fastest with 2-3 chunks at 8192^3 on B200: 5.23 ms per call against 5.48
  // with 8 chunks and 5.20 with the GEMMs left out.  More chunks only start
  // the first copy-out sooner, which a single unoverlapped call gains from.
  const int tiles_m = (M + kTileM - 1) / kTileM;
  const int want = whole ? 1 : (tiles_m < 3 ? tiles_m : 3);
  const int chunk_tiles = (tiles_m + want - 1) / want;
  const int chunk_rows = chunk_tiles * kTileM;
  const int chunks = (M + chunk_rows - 1) / chunk_rows;
  if (chunks > HostStaging::kMaxChunks) return B200GEMM_ERR_TOO_LARGE;

  auto ok = [](cudaError_t e) { return e == cudaSuccess; };
  // This set was last used by the call two back: the uploads wait for its
  // last GEMM, the GEMMs (which write dC) for its last copy-out.  A
  // never-recorded event is already complete.
  if (!ok(cudaStreamWaitEvent(st.s_h2d, buf.ev_read, 0)) || !ok(cudaStreamWaitEvent(st.s_mma, buf.ev_done, 0)))
    return B200GEMM_ERR_CUDA;
  auto* dA = static_cast<uint8_t*>(buf.dA);
  auto* dC = static_cast<uint8_t*>(buf.dC);
  const auto* srcA = static_cast<const uint8_t*>(hA);
  auto* dstC = static_cast<uint8_t*>(hC);
  auto enqueue = [&]() -> int {
    if (!ok(cudaEventRecord(st.ev_start, stream)) || !ok(cudaStreamWaitEvent(st.s_h2d, st.ev_start, 0)) ||
        !ok(cudaStreamWaitEvent(st.s_mma, st.ev_start, 0)) ||
        !ok(cudaStreamWaitEvent(st.s_d2h, st.ev_start, 0))) {
      return B200GEMM_ERR_CUDA;
    }
    if (bytesB > 0 && !ok(cudaMemcpyAsync(buf.dB, hB, bytesB, cudaMemcpyHostToDevice, st.s_h2d)))
      return B200GEMM_ERR_CUDA;
    if (!ok(cudaEventRecord(st.ev_b, st.s_h2d)) || !ok(cudaStreamWaitEvent(st.s_mma, st.ev_b, 0)))
      return B200GEMM_ERR_CUDA;
    for (int i = 0; i < chunks; ++i) {
      const int r0 = i * chunk_rows;
      const int rows = (M - r0) < chunk_rows ? (M - r0) : chunk_rows;
      const size_t a_off = static_cast<size_t>(r0) * K * 2;
      if (K > 0 && !ok(cudaMemcpyAsync(dA + a_off, srcA + a_off, static_cast<size_t>(rows) * K * 2,
                                       cudaMemcpyHostToDevice, st.s_h2d)))
        return B200GEMM_ERR_CUDA;
      if (!ok(cudaEventRecord(st.ev_a[i], st.s_h2d)) ||
          !ok(cudaStreamWaitEvent(st.s_mma, st.ev_a[i], 0)))
        return B200GEMM_ERR_CUDA;
      const int rc = gemm_device(h, rows, N, K, dA + a_off, buf.dB, dC + r0 * ldc_dev * 2,
                                 static_cast<int>(ldc_dev), st.s_mma, /*allow_small_m=*/whole);
      if (rc != B200GEMM_OK) return rc;
      if (!ok(cudaEventRecord(st.ev_c[i], st.s_mma)) ||
          !ok(cudaStreamWaitEvent(st.s_d2h, st.ev_c[i], 0)) ||
          !ok(cudaMemcpy2DAsync(dstC + static_cast<size_t>(r0) * ldc * 2, static_cast<size_t>(ldc) * 2,
                                dC + r0 * ldc_dev * 2, ldc_dev * 2, static_cast<size_t>(N) * 2,
                                static_cast<size_t>(rows), cudaMemcpyDeviceToHost, st.s_d2h)))
        return B200GEMM_ERR_CUDA;
    }
    return B200GEMM_OK;
  };
  const int rc = enqueue();
  // Whatever was enqueued, the set is reused only after it: record its
  // events on every path (a failed call leaves the caller's stream alone).
  const bool marked = ok(cudaEventRecord(buf.ev_read, st.s_mma)) && ok(cudaEventRecord(buf.ev_done, st.s_d2h));
  if (rc != B200GEMM_OK) return rc;
  if (!marked || !ok(cudaStreamWaitEvent(stream, buf.ev_done, 0))) return B200GEMM_ERR_CUDA;
  return B200GEMM_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot call cudaMalloc (or anything that allocates device
// memory) on the path that runs a GEMM: a memory-pool or caching-allocator
// implementation that calls the GEMM from inside its own bookkeeping, a
// serving process that plans all device memory at start-up and must not
// allocate afterwards (an allocation can block on the device, fail under
// fragmentation, or invalidate the plan), or code that cannot own a handle.
// b200gemm_bf16_nt_noalloc serves them: the caller passes A, B and C, and the
// only other device memory it touches is the fixed array below, compiled into
// this library.  Every GPU that loads the library holds the array until the
// process exits.
namespace {

constexpr uint32_t kNoAllocStatusWords = 64;   // 4 used; pads the table to a 256-byte boundary
constexpr uint32_t kNoAllocMaxTiles = 16384;   // largest tile grid one call may use

struct NoAllocDevice {
  bool ready = false;
  uint32_t* scratch = nullptr;  // device address of no_alloc_scratch on this device
  int clusters_n256 = 0;
  int clusters_n512 = 0;
};

constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice no_alloc_devices[kNoAllocMaxDevices];
std::mutex no_alloc_mu;

}  // namespace

// Status words followed by the tile schedule of the most recent call, shared
// by every call on the device.  In host code this name only stands for the
// symbol; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint32_t no_alloc_scratch[kNoAllocStatusWords + kNoAllocMaxTiles];

extern "C" int b200gemm_bf16_nt_noalloc(int M, int N, int K, const void* A, const void* B, void* C,
                                        int ldc, void* stream_ptr) {
  if (M < 0 || N < 0 || K < 0) return B200GEMM_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return B200GEMM_OK;
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr))) return B200GEMM_ERR_INVALID_ARG;
  if (ldc < N || (ldc % 8) != 0 || (K % 8) != 0) return B200GEMM_ERR_UNSUPPORTED;
  if (!aligned16(C) || (K > 0 && (!aligned16(A) || !aligned16(B)))) return B200GEMM_ERR_UNSUPPORTED;
  const uint32_t tiles_m = static_cast<uint32_t>((M + kTileM - 1) / kTileM);
  if (tiles_m > 0xFFFFu || static_cast<uint32_t>((N + kBlockN - 1) / kBlockN) > 0xFFFFu)
    return B200GEMM_ERR_TOO_LARGE;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200GEMM_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return B200GEMM_ERR_NO_DEVICE;
  NoAllocDevice st;
  {
    // One-time set-up per device, on the first call with that device current.
    std::lock_guard<std::mutex> lock(no_alloc_mu);
    NoAllocDevice& d = no_alloc_devices[dev];
    if (!d.ready) {
      int major = 0, minor = 0, sms = 0;
      if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        return B200GEMM_ERR_CUDA;
      }
      if (major != 10 || minor != 0) return B200GEMM_ERR_NO_DEVICE;
      if (tensor_map_encoder() == nullptr) return B200GEMM_ERR_CUDA;
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, no_alloc_scratch) != cudaSuccess || ptr == nullptr) {
        cudaGetLastError();
        return B200GEMM_ERR_CUDA;
      }
      const int c256 = prepare_kernel<CfgN256>(sms);
      const int c512 = prepare_kernel<CfgN512>(sms);
      if (c256 <= 0 || c512 <= 0) return B200GEMM_ERR_CUDA;
      // Load the schedule kernel's module now as well: with lazy module
      // loading its first launch would otherwise load it, which can allocate
      // device memory, on whichever later call first reaches that launch.
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, build_schedule_kernel) != cudaSuccess) {
        cudaGetLastError();
        return B200GEMM_ERR_CUDA;
      }
      d.scratch = static_cast<uint32_t*>(ptr);
      d.clusters_n256 = c256;
      d.clusters_n512 = c512;
      d.ready = true;
    }
    st = d;
  }

  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (K == 0) {  // empty sum: C = 0
    return cudaMemset2DAsync(C, static_cast<size_t>(ldc) * 2, 0, static_cast<size_t>(N) * 2,
                             static_cast<size_t>(M), stream) == cudaSuccess
               ? B200GEMM_OK
               : B200GEMM_ERR_CUDA;
  }

  const int num_kb = (K + kBlockK - 1) / kBlockK;
  const int width = tile_plan_cost(512, tiles_m, N, num_kb, st.clusters_n512) <
                            tile_plan_cost(256, tiles_m, N, num_kb, st.clusters_n256)
                        ? 512
                        : 256;
  const uint32_t tiles_n = static_cast<uint32_t>((N + width - 1) / width);
  const uint64_t tiles = static_cast<uint64_t>(tiles_m) * tiles_n;
  if (tiles > kNoAllocMaxTiles) return B200GEMM_ERR_TOO_LARGE;  // beyond the static table

  CUtensorMap ma, mb, mc;
  const uint64_t k = static_cast<uint64_t>(K);
  if (!encode_2d(&ma, A, k, static_cast<uint64_t>(M), k * 2, kBlockK, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&mb, B, k, static_cast<uint64_t>(N), k * 2, kBlockK, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&mc, C, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                 static_cast<uint64_t>(ldc) * 2, kCBoxCols, kCBoxRows, CU_TENSOR_MAP_SWIZZLE_64B)) {
    return B200GEMM_ERR_CUDA;
  }

  // The array keeps the previous call's contents: the status words must
  // start at zero and the schedule is rewritten for this tile grid.
  uint32_t* status = st.scratch;
  uint32_t* table = st.scratch + kNoAllocStatusWords;
  if (cudaMemsetAsync(status, 0, 4 * sizeof(uint32_t), stream) != cudaSuccess) return B200GEMM_ERR_CUDA;
  build_schedule_kernel<<<1, 1024, 0, stream>>>(tiles_m, tiles_n, B200GEMM_DEFAULT_ORDER,
                                                B200GEMM_DEFAULT_BAND, table);
  if (cudaGetLastError() != cudaSuccess) return B200GEMM_ERR_CUDA;

  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_kb = num_kb;
  p.num_tiles = static_cast<int>(tiles);
  p.num_units = p.num_tiles;  // no K-split tail on this path
  p.tail_start = p.num_tiles;
  p.tail_split = 1;
  p.tail_kb = num_kb;
  p.workspace = nullptr;
  p.tail_counters = nullptr;
  p.tiles = table;
  p.status = status;
  p.timeout_ns = kDefaultTimeoutNs;
  p.C = static_cast<uint16_t*>(C);
  p.ldc = ldc;
  p.npeers = 0;
  cudaError_t e;
  if (width == 512) {
    const int clusters = p.num_tiles < st.clusters_n512 ? p.num_tiles : st.clusters_n512;
    e = launch_gemm<CfgN512>(clusters, stream, ma, mb, mc, p);
  } else {
    const int clusters = p.num_tiles < st.clusters_n256 ? p.num_tiles : st.clusters_n256;
    e = launch_gemm<CfgN256>(clusters, stream, ma, mb, mc, p);
  }
  return e == cudaSuccess ? B200GEMM_OK : B200GEMM_ERR_CUDA;
}
