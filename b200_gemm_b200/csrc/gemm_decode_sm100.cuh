// Small-M ("decode") GEMM for sm_100a: C[M x N] = A[M x K] . B[N x K]^T with
// M <= 256, where streaming B from HBM is the whole cost (at M = 128,
// N = K = 8192, B is 128 MB and A is 2 MB).
//
// The tiled kernel (gemm_sm100.cuh) gives a CTA pair 256 rows of C, so at
// M = 128 half of every MMA is padding and only N / 256 pairs (32 of 74 at
// N = 8192) have work.  Here the operands swap roles: rows of B are the MMA's
// M side and the (at most 128, or 256) rows of A its N side, so a pair covers 256
// rows of B against all of A, and K is split across the S pairs of a
// cluster of 2S CTAs.  Each CTA pair accumulates its K range in TMEM
// (D[i][j] = sum_k B[n0 + i][k] * A[j][k] = C[j][n0 + i]); the pairs then
// exchange fp32 partial sums through distributed shared memory (st.async,
// counted on the receiver's mbarrier; a partial slice is stored as
// [column group of 4][B row][4 floats], so the 32 lanes of a warp, which hold
// 32 consecutive B rows, write 512 contiguous bytes per store and read them
// back bank-conflict free): CTA (pair p, half q) keeps the slice of
// A rows j in [p * NT/S, (p+1) * NT/S), receives the other pairs' partials
// of that slice, adds them, rounds to bf16 and writes C through a transposing
// staging buffer.  No global workspace, one launch, N/256 * 2S CTAs.
//
// Small shapes with more rows of A (up to a few thousand, few output tiles)
// run the same kernel over blocks of NT rows of A: one cluster per 256 rows
// of B x NT rows of A, N/256 * M/NT clusters, so K splits across the CTA
// pairs where the tiled kernel's few tiles would leave most SMs idle.
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


struct DecodeParams {
  int M, N, K;
  int num_kb;        // ceil(K / 64)
  int kb_per_split;  // K blocks per CTA pair, a multiple of the instance's kKps
  unsigned int* status;
  unsigned long long timeout_ns;
  EpiArgs epi;       // fused epilogue (identity: no flags, act none, bf16, alpha 1)
  int pdl;           // launch overlap with the previous kernel: kPdl*
  // Clusters are laid out [M block][N block]: cluster c covers rows of B
  // (columns of C) from 256 (c % n_blocks) and rows of A (rows of C) from
  // NT (c / n_blocks).  More than one M block (M > NT) needs slices that end
  // inside their block: split 1, 2 or 4.
  int n_blocks;      // ceil(N / 256)
};

// NT = rows of A covered (the MMA's N): 128 for M <= 128, 256 for M <= 256.
template <int S, int NT = 128>
struct DecodeCfg {
  static_assert(S == 1 || S == 2 || S == 3 || S == 4, "split factor");
  static_assert(NT == 128 || NT == 256, "rows of A per MMA");
  static_assert(S != 3 || NT == 256, "a split of 3 slices 256 rows of A as 96 + 96 + 64");
  static constexpr int kSplit = S;
  static constexpr int kNT = NT;
  static constexpr int kClusterSize = 2 * S;
  static constexpr int kThreads = 192;             // warps: 0 TMA, 1 MMA, 2-5 epilogue
  // With NT = 128 a stage holds 2 consecutive K blocks, requested back to
  // back, so each row of B is read 256 contiguous bytes at a time (measured:
  // equal or up to 9% faster than one K block per stage, most where few SMs
  // stream).  NT = 256 doubles A's share and its partial sums, leaving room
  // for one K block per stage.
  static constexpr int kKps = NT == 128 ? 2 : 1;
  static constexpr int kSubB = 128 * kBlockK * 2;             // 16 KB: this CTA's 128 rows of B, one K block
  static constexpr int kSubA = (kNT / 2) * kBlockK * 2;       // this CTA's NT/2 rows of A, one K block
  static constexpr int kStageB = kKps * kSubB;
  static constexpr int kStageA = kKps * kSubA;
  static constexpr int kStageBytes = kStageB + kStageA;
  // Rows of C (rows of A) each CTA pair finishes: kSliceRows for every pair
  // but the last, which takes the rest (S = 3: 96, 96, 64).  Slices are
  // whole 32-row chunks, and only the last may be shorter, so a C or residual
  // box of kSliceRows rows from the last slice's first row overhangs only
  // rows >= 256 >= M, which TMA clips (stores) or zero-fills (loads).
  static constexpr int kSliceRows = (kNT / S + 31) / 32 * 32;
  static constexpr int kLastSliceRows = kNT - (S - 1) * kSliceRows;
  static_assert(kLastSliceRows > 0 && kLastSliceRows <= kSliceRows && kLastSliceRows % 32 == 0, "slices");
  static constexpr int kRecvSlotBytes = 128 * kSliceRows * 4;  // [kSliceRows/4][128 rows][4] fp32
  static constexpr int kRecvBytes = (S - 1) * kRecvSlotBytes;
  static constexpr int kCWarpBytes = kSliceRows * 32 * 4;    // kSliceRows x 32 outputs (up to fp32) per warp
  static constexpr int kRWarpBytes = kSliceRows * 32 * 2;    // the same rows of the residual (bf16)
  static constexpr int kBarBytes = 256;
  // The ring takes every byte left: its depth is what hides HBM latency.
  static constexpr int kStagesFit = (232448 - 1024 - kBarBytes - kRecvBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 10 ? 10 : kStagesFit;
  static_assert(kStages >= 3, "pipeline too shallow");
  static_assert(4 * (kCWarpBytes + kRWarpBytes) <= kStages * kStageBytes,
                "C staging and residual tiles alias the operand ring");
  static constexpr int kB = 0;       // B stages, then A stages; after the last MMA the ring holds C staging
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((static_cast<uint32_t>(NT) >> 3) << 17) |
                                     ((256u >> 4) << 24);
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

// Instruction descriptor (DecodeCfg::kIdesc): kind::f16, D f32, A = B =
// bf16 K-major, M = 256 (pair), N = NT.

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    gemm_bf16_nt_decode_sm100(const __grid_constant__ CUtensorMap map_a,
                              const __grid_constant__ CUtensorMap map_b,
                              const __grid_constant__ CUtensorMap map_c,
                              const __grid_constant__ CUtensorMap map_r, const DecodeParams p) {
  constexpr int S = Cfg::kSplit;
  constexpr int STAGES = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t rank = ptx::cluster_ctarank();
  const uint32_t pair = rank >> 1, half = rank & 1u;
  auto slice_rows = [](uint32_t pr) {
    return pr + 1 == static_cast<uint32_t>(S) ? Cfg::kLastSliceRows : Cfg::kSliceRows;
  };
  const bool leader = half == 0;
  const int n0 = static_cast<int>(ptx::cluster_id_x() % static_cast<uint32_t>(p.n_blocks)) * 256;
  const int m0 = static_cast<int>(ptx::cluster_id_x() / static_cast<uint32_t>(p.n_blocks)) * Cfg::kNT;
  const int kb_begin = static_cast<int>(pair) * p.kb_per_split;
  const int kb_end = min(p.num_kb, kb_begin + p.kb_per_split);
  const int nkb = kb_end > kb_begin ? kb_end - kb_begin : 0;

  const uint32_t sB = base + Cfg::kB, sA = base + Cfg::kA, sRecv = base + Cfg::kRecv;
  const uint32_t sC = sB;  // C staging reuses the operand ring once the MMAs are done
  const uint32_t full0 = base + Cfg::kFull, empty0 = base + Cfg::kEmpty;
  const uint32_t tfull = base + Cfg::kTFull, recv_bar = base + Cfg::kRecvBar;
  const uint32_t drain = base + Cfg::kDrain, tmem_slot = base + Cfg::kTmemSlot;

  ptx::Watchdog wd;
  wd.abort_flag = base + Cfg::kAbort;
  wd.peer_abort_flag = ptx::mapa(wd.abort_flag, rank ^ 1u);
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
    // The partner pairs' partial slices arrive as counted bytes; the one
    // arrival is this expect_tx, made before any partner can send.
    if (S > 1) ptx::mbar_arrive_expect_tx(recv_bar, (S - 1) * 128 * 4 * slice_rows(pair));
    ptx::prefetch_tensormap(&map_a);
    ptx::prefetch_tensormap(&map_b);
    ptx::prefetch_tensormap(&map_c);
    if (p.epi.flags & kEpiResidual) ptx::prefetch_tensormap(&map_r);
  }
  if (warp == 1) {
    ptx::tmem_alloc_cg2(tmem_slot, Cfg::kNT);
    ptx::tmem_relinquish_cg2();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync_all();
  ptx::tc_fence_after();
  uint32_t tmem_base;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem_base) : "r"(tmem_slot) : "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nkb > 0) {
      const uint64_t policy_b = ptx::policy_evict_first();  // B is read once
      const uint64_t policy_a = ptx::policy_evict_last();   // A is read by every cluster
      const uint32_t full_leader0 = ptx::mapa(full0, rank & ~1u);
      // With kPdlWeightsEarly the first ring of B (the weights, which the
      // previous kernel does not write) streams in before that kernel has
      // finished; A and everything after wait for it.
      // Each stage covers K blocks [kb, kb + KPS); the pair's range is a whole
      // number of stages (a block past K reads as zeros).
      constexpr int KPS = Cfg::kKps;
      const int brow = n0 + static_cast<int>(half) * 128, arow = m0 + static_cast<int>(half) * (Cfg::kNT / 2);
      const int nst = (nkb + KPS - 1) / KPS;
      const int pre = p.pdl == kPdlWeightsEarly ? min(STAGES, nst) : 0;
      for (int s = 0; s < pre; ++s) {
        if (leader) ptx::mbar_arrive_expect_tx(full0 + 8 * s, 2 * Cfg::kStageBytes);
#pragma unroll
        for (int j = 0; j < KPS; ++j)
          ptx::tma_load_2d_cg2(sB + s * Cfg::kStageB + j * Cfg::kSubB, &map_b, full_leader0 + 8 * s,
                               (kb_begin + s * KPS + j) * kBlockK, brow, policy_b);
      }
      ptx::griddep_wait();
      for (int s = 0; s < pre; ++s) {
#pragma unroll
        for (int j = 0; j < KPS; ++j)
          ptx::tma_load_2d_cg2(sA + s * Cfg::kStageA + j * Cfg::kSubA, &map_a, full_leader0 + 8 * s,
                               (kb_begin + s * KPS + j) * kBlockK, arow, policy_a);
      }
      uint32_t stage = pre == STAGES ? 0u : static_cast<uint32_t>(pre);
      uint32_t phase = pre == STAGES ? 1u : 0u;
      for (int kb = kb_begin + pre * KPS; kb < kb_end; kb += KPS) {
        if (!ptx::mbar_wait(empty0 + 8 * stage, phase ^ 1u, wd, kSiteProducer, 0)) break;
        if (leader) ptx::mbar_arrive_expect_tx(full0 + 8 * stage, 2 * Cfg::kStageBytes);
        const uint32_t fb = full_leader0 + 8 * stage;
#pragma unroll
        for (int j = 0; j < KPS; ++j)
          ptx::tma_load_2d_cg2(sB + stage * Cfg::kStageB + j * Cfg::kSubB, &map_b, fb, (kb + j) * kBlockK, brow,
                               policy_b);
#pragma unroll
        for (int j = 0; j < KPS; ++j)
          ptx::tma_load_2d_cg2(sA + stage * Cfg::kStageA + j * Cfg::kSubA, &map_a, fb, (kb + j) * kBlockK, arow,
                               policy_a);
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
    if (leader && lane == 0) {
      const uint32_t own_empty0 = ptx::mapa(empty0, rank), peer_empty0 = ptx::mapa(empty0, rank + 1);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; kb += Cfg::kKps) {
        if (!ptx::mbar_wait(full0 + 8 * stage, phase, wd, kSiteMmaFull, 0)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
#pragma unroll
        for (int j = 0; j < Cfg::kKps; ++j) {
          const uint64_t a_desc = smem_desc(sB + stage * Cfg::kStageB + j * Cfg::kSubB);  // MMA A: rows of B
          const uint64_t b_desc = smem_desc(sA + stage * Cfg::kStageA + j * Cfg::kSubA);  // MMA B: rows of A
#pragma unroll
          for (int k = 0; k < kBlockK / kMmaK; ++k) {
            ptx::mma_bf16_cg2(tmem_base, a_desc + 2 * k, b_desc + 2 * k, Cfg::kIdesc,
                              (kb > kb_begin || j > 0 || k > 0) ? 1u : 0u);
          }
        }
        ptx::mma_commit_cg2(own_empty0 + 8 * stage);
        ptx::mma_commit_cg2(peer_empty0 + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        ptx::mma_commit_cg2(ptx::mapa(tfull, rank));
        ptx::mma_commit_cg2(ptx::mapa(tfull, rank + 1));
      }
      ptx::mma_commit_cg2(ptx::mapa(drain, rank));
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
    const bool have = nkb > 0;                      // a pair with no K blocks contributes zeros
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
    const int row0 = m0 + static_cast<int>(pair) * Cfg::kSliceRows;
    const int col = n0 + static_cast<int>(half) * 128 + static_cast<int>(quarter) * 32;
    const uint32_t res_bar = base + Cfg::kResBar + 8 * (warp - 2u);
    const uint32_t rtile = sC + 4 * Cfg::kCWarpBytes + (warp - 2u) * Cfg::kRWarpBytes;
    const bool res_load = ok && (p.epi.flags & kEpiResidual) && row0 < p.M && col < p.N;
    if (res_load && lane == 0) {
      ptx::mbar_arrive_expect_tx(res_bar, Cfg::kRWarpBytes);
      ptx::tma_load_2d(rtile, &map_r, res_bar, col, row0, ptx::policy_evict_first());
    }
    // 1. Send the slices that other pairs finish.
    if (ok && S > 1) {
#pragma unroll 1
      for (int dst_pair = 0; dst_pair < S; ++dst_pair) {
        if (dst_pair == static_cast<int>(pair)) continue;
        const uint32_t dst_cta = static_cast<uint32_t>(dst_pair) * 2u + half;
        const int slot = static_cast<int>(pair) < dst_pair ? static_cast<int>(pair) : static_cast<int>(pair) - 1;
        const uint32_t remote_row = ptx::mapa(sRecv + slot * Cfg::kRecvSlotBytes + i * 16u, dst_cta);
        const uint32_t remote_bar = ptx::mapa(recv_bar, dst_cta);
#pragma unroll 1
        for (int c = 0; c < slice_rows(static_cast<uint32_t>(dst_pair)) / 32; ++c) {
          uint32_t v[32];
          if (have) {
            ptx::tmem_ld_32x32b_x32(t_row + dst_pair * Cfg::kSliceRows + c * 32, v);
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
    if (early_ld) ptx::tmem_ld_32x32b_x32(t_row + pair * Cfg::kSliceRows, v);
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
      for (int c = 0; c < slice_rows(pair) / 32; ++c) {
        if (have) {
          if (c > 0 || S == 1) ptx::tmem_ld_32x32b_x32(t_row + pair * Cfg::kSliceRows + c * 32, v);
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
  if (warp == 1) ptx::tmem_dealloc_cg2(tmem_base, Cfg::kNT);
}

}  // namespace b200gemm
