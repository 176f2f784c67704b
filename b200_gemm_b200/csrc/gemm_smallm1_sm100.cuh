// Small-M GEMM, single-CTA form (cta_group::1), for sm_100a:
// C[M x N] = A[M x K] . B[N x K]^T with M <= 128.  Like the pair kernel of
// gemm_decode_sm100.cuh the operands swap roles (rows of B are the MMA's M
// side, all rows of A its N side) and streaming B from HBM is the whole
// cost, but here each CTA alone covers 128 rows of B (MMA 128 x 128 x 16),
// so a shape gets twice the CTAs of the pair kernel for the same K split.
// That is what narrow N needs: one SM's share of HBM bandwidth is bounded by
// the bytes its shared-memory ring keeps in flight, so N = 4096 (16 pairs of
// 256 rows) must be spread over more SMs than the pair kernel's clusters of
// 8 CTAs can co-reside on (15 of them fit on a 148-SM B200).
//
// A cluster of S CTAs (S = 1, 2, 4) splits K; CTA r accumulates its K range
// in TMEM (D[i][j] = sum_k B[n0 + i][k] * A[j][k] = C[j][n0 + i]), then the
// CTAs exchange fp32 partials through distributed shared memory (st.async,
// counted on the receiver's mbarrier): CTA r keeps A rows
// j in [r * 128/S, (r+1) * 128/S), adds the other CTAs' partials of that
// slice, rounds to bf16 and writes C through a transposing staging buffer.
//
// Reference path: b200_kernels/matmul_1.cuh:329-418 computes the same C with
// 256 x 256 tiles only; decode shapes are a benchmark configuration the
// reference does not specialise.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "gemm_sm100.cuh"

namespace b200gemm {

struct SmallMParams {
  int M, N, K;
  int num_kb;        // ceil(K / 64)
  int kb_per_split;  // K blocks per CTA
  unsigned int* status;
  unsigned long long timeout_ns;
  EpiArgs epi;       // fused epilogue (identity: no flags, act none, bf16, alpha 1)
  int pdl;           // launch overlap with the previous kernel: kPdl*
};

template <int S>
struct SmallMCfg {
  static_assert(S == 1 || S == 2 || S == 4, "split factor");
  static constexpr int kSplit = S;
  static constexpr int kRowsB = 128;               // rows of B per CTA (MMA M)
  static constexpr int kNT = 128;                  // rows of A covered (MMA N)
  static constexpr int kThreads = 192;             // warps: 0 TMA, 1 MMA, 2-5 epilogue
  static constexpr int kStageB = kRowsB * kBlockK * 2;       // 16 KB
  static constexpr int kStageA = kNT * kBlockK * 2;          // 16 KB
  static constexpr int kStageBytes = kStageB + kStageA;
  static constexpr int kSliceRows = kNT / S;                 // rows of C each CTA finishes
  static constexpr int kRecvSlotBytes = kRowsB * kSliceRows * 4;  // [kSliceRows/4][128 rows][4] fp32
  static constexpr int kRecvBytes = (S - 1) * kRecvSlotBytes;
  static constexpr int kCWarpBytes = kSliceRows * 32 * 4;    // kSliceRows x 32 outputs (up to fp32) per warp
  static constexpr int kRWarpBytes = kSliceRows * 32 * 2;    // the same rows of the residual (bf16)
  static constexpr int kBarBytes = 256;
  static constexpr int kStagesFit = (232448 - 1024 - kBarBytes - kRecvBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static_assert(kStages >= 4, "pipeline too shallow");
  static_assert(4 * (kCWarpBytes + kRWarpBytes) <= kStages * kStageB, "C staging and residual tiles alias the B stages");
  static constexpr int kB = 0;       // B stages; after the last MMA they hold the C staging buffers
  static constexpr int kA = kB + kStages * kStageB;
  static constexpr int kRecv = kA + kStages * kStageA;
  static constexpr int kFull = kRecv + kRecvBytes;
  static constexpr int kEmpty = kFull + 8 * kStages;
  static constexpr int kTFull = kEmpty + 8 * kStages;
  static constexpr int kResBar = kTFull + 8;   // one per epilogue warp: its residual tile landed
  static constexpr int kRecvBar = kResBar + 32;
  static constexpr int kDrain = kRecvBar + 8;
  static constexpr int kTmemSlot = kDrain + 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kEnd = kAbort + 4;
  static_assert(kEnd - kFull <= kBarBytes, "barrier area");
  static constexpr int kSmemBytes = kEnd + 1024;
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
};

// kind::f16, D f32, A = B = bf16 K-major, M = 128, N = 128.
constexpr uint32_t kIdescSmallM1 = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) |
                                   ((128u >> 4) << 24);

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    gemm_bf16_nt_smallm1_sm100(const __grid_constant__ CUtensorMap map_a,
                               const __grid_constant__ CUtensorMap map_b,
                               const __grid_constant__ CUtensorMap map_c,
                               const __grid_constant__ CUtensorMap map_r, const SmallMParams p) {
  constexpr int S = Cfg::kSplit;
  constexpr int STAGES = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t rank = S > 1 ? ptx::cluster_ctarank() : 0u;  // K slice of this CTA
  const int n0 = static_cast<int>(S > 1 ? ptx::cluster_id_x() : blockIdx.x) * Cfg::kRowsB;
  const int kb_begin = static_cast<int>(rank) * p.kb_per_split;
  const int kb_end = min(p.num_kb, kb_begin + p.kb_per_split);
  const int nkb = kb_end > kb_begin ? kb_end - kb_begin : 0;

  const uint32_t sB = base + Cfg::kB, sA = base + Cfg::kA, sRecv = base + Cfg::kRecv;
  const uint32_t sC = sB;  // C staging reuses the B stages once the MMAs are done
  const uint32_t full0 = base + Cfg::kFull, empty0 = base + Cfg::kEmpty;
  const uint32_t tfull = base + Cfg::kTFull, recv_bar = base + Cfg::kRecvBar;
  const uint32_t drain = base + Cfg::kDrain, tmem_slot = base + Cfg::kTmemSlot;

  ptx::Watchdog wd;
  wd.abort_flag = base + Cfg::kAbort;
  // A timeout is passed on to one other CTA of the cluster (the rest find
  // out through their own bounded waits); alone, the CTA flags itself.
  wd.peer_abort_flag = S > 1 ? ptx::mapa(wd.abort_flag, rank ^ 1u) : wd.abort_flag;
  wd.status = p.status;
  wd.timeout_ns = p.timeout_ns;

  if (threadIdx.x == 0) {
    asm volatile("st.shared.u32 [%0], 0;" ::"r"(wd.abort_flag) : "memory");
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full0 + 8 * s, 1);
      ptx::mbar_init(empty0 + 8 * s, 1);
    }
    ptx::mbar_init(tfull, 1);
    for (int w = 0; w < 4; ++w) ptx::mbar_init(base + Cfg::kResBar + 8 * w, 1);
    ptx::mbar_init(recv_bar, 1);
    ptx::mbar_init(drain, 1);
    ptx::fence_mbar_init_cluster();
    // The other CTAs' partial slices arrive as counted bytes; the one
    // arrival is this expect_tx, made before any of them can send.
    if (S > 1) ptx::mbar_arrive_expect_tx(recv_bar, Cfg::kRecvBytes);
    ptx::prefetch_tensormap(&map_a);
    ptx::prefetch_tensormap(&map_b);
    ptx::prefetch_tensormap(&map_c);
    if (p.epi.flags & kEpiResidual) ptx::prefetch_tensormap(&map_r);
  }
  if (warp == 1) {
    ptx::tmem_alloc_cg1(tmem_slot, Cfg::kNT);
    ptx::tmem_relinquish_cg1();
  }
  // The producer's loads signal only this CTA's barriers (initialised above
  // by this same thread), so the first ring of them goes out between the
  // two halves of the cluster barrier instead of after the whole prologue.
  const uint64_t policy_b = ptx::policy_evict_first();  // B is read once
  const uint64_t policy_a = ptx::policy_evict_last();   // A is read by every cluster
  const int early = nkb < STAGES ? nkb : STAGES;
  ptx::tc_fence_before();
  ptx::cluster_arrive();
  if (warp == 0 && lane == 0) {
    // With kPdlWeightsEarly B (the weights, which the previous kernel does
    // not write) streams in before that kernel has finished; A waits for it.
    const bool b_first = p.pdl == kPdlWeightsEarly;
    if (!b_first) ptx::griddep_wait();
    for (int s = 0; s < early; ++s) {
      const int kb = kb_begin + s;
      ptx::mbar_arrive_expect_tx(full0 + 8 * s, Cfg::kStageBytes);
      ptx::tma_load_2d(sB + s * Cfg::kStageB, &map_b, full0 + 8 * s, kb * kBlockK, n0, policy_b);
      if (!b_first) ptx::tma_load_2d(sA + s * Cfg::kStageA, &map_a, full0 + 8 * s, kb * kBlockK, 0, policy_a);
    }
    if (b_first) {
      ptx::griddep_wait();
      for (int s = 0; s < early; ++s)
        ptx::tma_load_2d(sA + s * Cfg::kStageA, &map_a, full0 + 8 * s, (kb_begin + s) * kBlockK, 0, policy_a);
    }
  }
  ptx::cluster_wait();
  ptx::tc_fence_after();
  uint32_t tmem_base;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem_base) : "r"(tmem_slot) : "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nkb > early) {
      uint32_t stage = early == STAGES ? 0u : static_cast<uint32_t>(early);
      uint32_t phase = early == STAGES ? 1u : 0u;
      for (int kb = kb_begin + early; kb < kb_end; ++kb) {
        if (!ptx::mbar_wait(empty0 + 8 * stage, phase ^ 1u, wd, kSiteProducer, 0)) break;
        ptx::mbar_arrive_expect_tx(full0 + 8 * stage, Cfg::kStageBytes);
        ptx::tma_load_2d(sB + stage * Cfg::kStageB, &map_b, full0 + 8 * stage, kb * kBlockK, n0, policy_b);
        ptx::tma_load_2d(sA + stage * Cfg::kStageA, &map_a, full0 + 8 * stage, kb * kBlockK, 0, policy_a);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
    if (p.pdl != kPdlOff) ptx::griddep_launch_dependents();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!ptx::mbar_wait(full0 + 8 * stage, phase, wd, kSiteMmaFull, 0)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint64_t a_desc = smem_desc(sB + stage * Cfg::kStageB);  // MMA A operand: rows of B
        const uint64_t b_desc = smem_desc(sA + stage * Cfg::kStageA);  // MMA B operand: rows of A
#pragma unroll
        for (int k = 0; k < kBlockK / kMmaK; ++k) {
          ptx::mma_bf16_cg1(tmem_base, a_desc + 2 * k, b_desc + 2 * k, kIdescSmallM1,
                            (kb > kb_begin || k > 0) ? 1u : 0u);
        }
        ptx::mma_commit_cg1(empty0 + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok && nkb > 0) ptx::mma_commit_cg1(tfull);
      // Every MMA issued here must be complete before TMEM is freed.
      ptx::mma_commit_cg1(drain);
      ptx::Watchdog dwd = wd;
      dwd.timeout_ns = 100000000ull;
      ptx::mbar_wait_drain(drain, 0, dwd, kSiteDrain);
    }
    __syncwarp();
    if (p.pdl != kPdlOff) ptx::griddep_launch_dependents();
  } else {
    // ------------------------------------------------------------ epilogue
    const uint32_t quarter = warp & 3u;             // TMEM lanes = rows of B this warp holds
    const uint32_t i = quarter * 32u + lane;        // this thread's row of B within the CTA
    const uint32_t t_row = tmem_base + ((quarter * 32u) << 16);
    const bool have = nkb > 0;                      // a CTA with no K blocks contributes zeros
    bool ok = true;
    ptx::griddep_wait();  // bias, residual and C may belong to the previous kernel
    if (have) {
      const bool got = ptx::mbar_wait(tfull, 0, wd, kSiteEpilogue, 0);
      ok = __all_sync(0xFFFFFFFFu, got);
      ptx::tc_fence_after();
    }
    if (p.pdl != kPdlOff) ptx::griddep_launch_dependents();
    // The residual rows and columns this warp adds at the end: one TMA load
    // into the B stages (free once the MMAs are done), in flight during the
    // exchange below.  Rows past M and columns past N read as zeros.
    const int row0 = static_cast<int>(rank) * Cfg::kSliceRows;
    const int col = n0 + static_cast<int>(quarter) * 32;
    const uint32_t res_bar = base + Cfg::kResBar + 8 * (warp - 2u);
    const uint32_t rtile = sC + 4 * Cfg::kCWarpBytes + (warp - 2u) * Cfg::kRWarpBytes;
    const bool res_load = ok && (p.epi.flags & kEpiResidual) && row0 < p.M && col < p.N;
    if (res_load && lane == 0) {
      ptx::mbar_arrive_expect_tx(res_bar, Cfg::kRWarpBytes);
      ptx::tma_load_2d(rtile, &map_r, res_bar, col, row0, ptx::policy_evict_first());
    }
    // 1. Send the slices that the other CTAs finish.
    if (ok && S > 1) {
#pragma unroll 1
      for (int dst = 0; dst < S; ++dst) {
        if (dst == static_cast<int>(rank)) continue;
        const int slot = static_cast<int>(rank) < dst ? static_cast<int>(rank) : static_cast<int>(rank) - 1;
        const uint32_t remote_row =
            ptx::mapa(sRecv + slot * Cfg::kRecvSlotBytes + i * 16u, static_cast<uint32_t>(dst));
        const uint32_t remote_bar = ptx::mapa(recv_bar, static_cast<uint32_t>(dst));
#pragma unroll 1
        for (int c = 0; c < Cfg::kSliceRows / 32; ++c) {
          uint32_t v[32];
          if (have) {
            ptx::tmem_ld_32x32b_x32(t_row + dst * Cfg::kSliceRows + c * 32, v);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(v);
          } else {
#pragma unroll
            for (int t = 0; t < 32; ++t) v[t] = 0u;
          }
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            ptx::st_async_v4(remote_row + static_cast<uint32_t>(c * 8 + g) * 2048u, remote_bar, v[4 * g],
                             v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
          }
        }
      }
    }
    // 2. Finish this CTA's slice: own partial + received partials -> bf16 -> C.
    // With a K split, the first 32 columns of the own partial are read from
    // TMEM while the partners' slices are still arriving.
    uint32_t v[32];
    const bool early_ld = S > 1 && ok && have;
    if (early_ld) ptx::tmem_ld_32x32b_x32(t_row + rank * Cfg::kSliceRows, v);
    if (ok && S > 1) {
      const bool got = ptx::mbar_wait(recv_bar, 0, wd, kSiteEpilogue, 1);
      ok = __all_sync(0xFFFFFFFFu, got);
      if (!ok && early_ld) ptx::tmem_wait_ld();  // no TMEM load left in flight
    }
    if (ok) {
      const uint32_t cw = sC + (warp - 2u) * Cfg::kCWarpBytes;  // [kSliceRows][32] outputs
      const bool epi_on = p.epi.flags != 0u || p.epi.act != kActNone || p.epi.alpha != 1.0f;
      if (res_load) {
        const bool got = ptx::mbar_wait(res_bar, 0, wd, kSiteEpilogue, 2);
        ok = __all_sync(0xFFFFFFFFu, got);
      }
#pragma unroll 1
      for (int c = 0; c < Cfg::kSliceRows / 32; ++c) {
        if (have) {
          if (c > 0 || S == 1) ptx::tmem_ld_32x32b_x32(t_row + rank * Cfg::kSliceRows + c * 32, v);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = 0u;
        }
        float acc[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[t] = __uint_as_float(v[t]);
#pragma unroll 1
        for (int slot = 0; slot < S - 1; ++slot) {
          const uint32_t row = sRecv + slot * Cfg::kRecvSlotBytes + i * 16u;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            uint32_t x0, x1, x2, x3;
            ptx::ld_shared_v4(row + static_cast<uint32_t>(c * 8 + g) * 2048u, x0, x1, x2, x3);
            acc[4 * g] += __uint_as_float(x0);
            acc[4 * g + 1] += __uint_as_float(x1);
            acc[4 * g + 2] += __uint_as_float(x2);
            acc[4 * g + 3] += __uint_as_float(x3);
          }
        }
        if (epi_on) smallm_epilogue(acc, col + static_cast<int>(lane), p.epi, p.N, rtile + c * 32 * 64 + lane * 2);
        // Transpose through shared memory: thread `lane` owns column `lane`
        // of the warp's 32-column block of C; rows are the slice's A rows.
        smallm_stage(acc, cw, c, lane, p.epi.out_type, p.epi.out_scale);
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < p.M && col < p.N) {
        ptx::tma_store_2d(&map_c, cw, col, row0);
        ptx::bulk_commit_group();
        ptx::bulk_wait_group_read<0>();  // smem reusable; the stores land before the kernel completes
      }
      __syncwarp();
    }
  }

  // --------------------------------------------------------------- teardown
  if (threadIdx.x == 0 && ptx::aborted(wd)) ptx::sleep_ns_bounded(200000ull);
  ptx::tc_fence_before();
  ptx::cluster_sync_all();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc_cg1(tmem_base, Cfg::kNT);
}

}  // namespace b200gemm
