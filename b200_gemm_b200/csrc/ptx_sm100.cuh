// sm_100a PTX building blocks for the bf16 GEMM: mbarriers with bounded
// waits, TMA tensor loads/stores, tcgen05 (TMEM alloc, MMA, commit, ld) and
// cluster helpers.  Every wrapper is a single PTX instruction (or a short
// fixed sequence) written from the PTX ISA description of that instruction.
//
// Role in the reference: these replace the helper layer of
// include/b200_utils.cuh (reference lines 18-514).  Differences that matter:
//   * every mbarrier wait is bounded by a %globaltimer budget and reports a
//     status instead of spinning forever (reference `wait`, lines 451-463);
//   * the leader-CTA barrier address comes from `mapa`, not from clearing
//     bit 24 of the shared address (reference `mbar_cta0_addr`, line 66);
//   * every TMA load here lands in the issuing CTA only (none is broadcast to
//     other CTAs of the cluster), so the library
//     is safe to run on every GPU of a multi-GPU job.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace b200gemm {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// Full cluster barrier (all threads of every CTA in the cluster).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The two halves of cluster_sync_all, for work that may run between them.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Programmatic dependent launch.  griddep_wait blocks the calling thread until
// the grids this one was launched to overlap with have completed and their
// memory is visible (it returns at once when there are none);
// griddep_launch_dependents lets a grid launched to overlap with this one be
// scheduled once every CTA of this grid has issued it or exited.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Arrive on an mbarrier that may live in another CTA of the cluster
// (`cluster_bar` is a shared::cluster address, e.g. from mapa()).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// ------------------------------------------------------------- watchdog
// Shared state for the bounded waits of one CTA.  When a wait runs out of
// budget the CTA (and its cluster peer) is flagged as aborted, a status code
// is published to global memory, and every other wait in the CTA returns
// false at its next poll instead of spinning.
struct Watchdog {
  uint32_t abort_flag;       // shared::cta address of this CTA's abort word
  uint32_t peer_abort_flag;  // shared::cluster address of the peer's abort word
  unsigned int* status;      // device status words [code, site, cluster, tile]
  uint64_t timeout_ns;
};

enum : unsigned int {
  kStatusOk = 0,
  kStatusTimeout = 4,  // matches B200GEMM_ERR_DEVICE_TIMEOUT
};

__device__ __forceinline__ bool aborted(const Watchdog& wd) {
  uint32_t v;
  asm volatile("ld.volatile.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(wd.abort_flag) : "memory");
  return v != 0;
}

__device__ __forceinline__ void raise_abort(const Watchdog& wd, unsigned int site, unsigned int tile) {
  asm volatile("st.volatile.shared::cta.u32 [%0], %1;" ::"r"(wd.abort_flag), "r"(1u) : "memory");
  asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(wd.peer_abort_flag), "r"(1u)
               : "memory");
  if (wd.status != nullptr) {
    if (atomicCAS(&wd.status[0], 0u, kStatusTimeout) == 0u) {
      wd.status[1] = site;
      wd.status[2] = cluster_id_x() * 2u + cluster_ctarank();
      wd.status[3] = tile;
      __threadfence();
    }
  }
}

// Wait for phase `parity` of an mbarrier.  Returns false (without hanging)
// when the budget runs out or another role of this cluster already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const Watchdog& wd,
                                          unsigned int site, unsigned int tile) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  // Iteration cap as a second bound in case the timer does not advance.
  const uint64_t max_iters = (wd.timeout_ns >> 2) + 1024;
  for (uint64_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 7) == 0) {
      if (aborted(wd)) return false;
      if (globaltimer_ns() - t0 > wd.timeout_ns || it > max_iters) {
        raise_abort(wd, site, tile);
        return false;
      }
    }
  }
}

// Bounded wait that ignores the abort word: used at teardown to wait for
// work this thread itself issued (e.g. MMAs still reading shared memory).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, const Watchdog& wd,
                                                unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t max_iters = (wd.timeout_ns >> 2) + 1024;
  for (uint64_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 7) == 0 && (globaltimer_ns() - t0 > wd.timeout_ns || it > max_iters)) {
      raise_abort(wd, site, 0xFFFFFFFFu);
      return false;
    }
  }
}

// Spin (bounded) for `ns` nanoseconds; used to let in-flight asynchronous
// copies land before an aborted CTA tears down.
__device__ __forceinline__ void sleep_ns_bounded(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    if (globaltimer_ns() - t0 > ns) break;
    __nanosleep(1000);
  }
}

// ------------------------------------------------------------------- TMA
// 2D tiled load into this CTA's shared memory; completion (bytes) is
// signalled on `cluster_bar`, which for cta_group::2 may be the barrier of
// the leader CTA of the pair.
__device__ __forceinline__ void tma_load_2d_cg2(uint32_t dst, const CUtensorMap* map,
                                                uint32_t cluster_bar, int x, int y,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 2D tiled load into this CTA's shared memory, completion (bytes) on this
// CTA's mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                            int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 eviction-priority policies for the cache_hint operand.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 0 = evict_normal, 1 = evict_last, 2 = evict_first
__device__ __forceinline__ uint64_t l2_policy(int kind) {
  return kind == 1 ? policy_evict_last() : (kind == 2 ? policy_evict_first() : policy_evict_normal());
}

// TMA store of a C tile.  Its L2 lines are marked evict_first: C is written
// once and not read back, so under L2 pressure its lines go before the
// operands' (measured: bit-identical output, 0.3-0.5% faster on the MLP
// shapes and 4096^3, unchanged at 8192^3).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y), "l"(policy_evict_first())
      : "memory");
}

// --------------------------------------------------------------- tcgen05
// TMEM allocation for a CTA pair: one warp of each CTA executes these.
__device__ __forceinline__ void tmem_alloc_cg2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_cg2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Single-CTA (cta_group::1) forms of the TMEM allocation, MMA and commit.
__device__ __forceinline__ void tmem_alloc_cg1(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_cg1() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_cg1(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void mma_bf16_cg1(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit_cg1(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T for a CTA pair, kind::f16 (bf16 inputs
// here, fp32 accumulate).  `accumulate` = 0 overwrites D.
__device__ __forceinline__ void mma_bf16_cg2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on one mbarrier (a shared::cluster address, so it may be
// the peer CTA's) when all previously issued tcgen05 async operations of
// this thread have completed.  Issuing it twice, once per CTA of the pair,
// signals both CTAs.
__device__ __forceinline__ void mma_commit_cg2(uint32_t cluster_bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          cluster_bar)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// lane (base_lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void reg_fence16(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Registers written by tcgen05.ld are only defined after tcgen05.wait::ld.
// Passing them through an empty volatile asm placed after the wait makes
// every later use depend on it, so no use can be scheduled above the wait.
__device__ __forceinline__ void reg_fence32(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

// Two fp32 -> packed bf16x2 with round-to-nearest-even (lo in bits 0-15).
__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo_f32, uint32_t hi_f32) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(hi_f32)),
      "f"(__uint_as_float(lo_f32)));
  return r;
}

// Four fp32 values -> four fp8 e4m3 bytes (RNE, saturated to +-448; NaN
// stays NaN), x0 in the lowest byte.
__device__ __forceinline__ uint32_t pack_e4m3x4(float x0, float x1, float x2, float x3) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(x1), "f"(x0));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(x3), "f"(x2));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// 16-byte store into another CTA's shared memory (shared::cluster address)
// whose completion is counted, in bytes, on an mbarrier of that CTA.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, uint32_t cluster_bar, uint32_t a,
                                            uint32_t b, uint32_t c, uint32_t d) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          cluster_addr),
      "r"(a), "r"(b), "r"(c), "r"(d), "r"(cluster_bar)
      : "memory");
}

__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                             uint32_t& d) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr)
               : "memory");
}

// 16-byte store to global memory (local or a peer GPU's, through its
// IPC/peer mapping).
__device__ __forceinline__ void st_global_v4(void* ptr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// 16-byte store through an NVLink multicast (NVLS) mapping: NVSwitch
// replicates it into the memory of every GPU bound to the multicast object.
// The words are stored as they are (a store does not interpret them).
__device__ __forceinline__ void multimem_st_v4(void* mc_ptr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_ptr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// 16-byte load cached in L2 only (data written by other SMs in this launch).
__device__ __forceinline__ void ld_global_cg_v4(const void* ptr, uint32_t& a, uint32_t& b, uint32_t& c,
                                                uint32_t& d) {
  asm volatile("ld.global.cg.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "l"(ptr)
               : "memory");
}

// Hint: bring the 128-byte line holding `ptr` into L2.
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// Hardware approximations (one MUFU operation each): tanh with relative
// error about 2^-11 and the reciprocal, both ISA instructions.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16-byte load of data that stays unchanged for the whole kernel (bias,
// residual) through the non-coherent path.
__device__ __forceinline__ void ld_global_nc_v4(const void* ptr, uint32_t& a, uint32_t& b, uint32_t& c,
                                                uint32_t& d) {
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "l"(ptr));
}

// 32-byte load (256-bit access; `ptr` 32-byte aligned), non-coherent path.
__device__ __forceinline__ void ld_global_nc_v8(const void* ptr, uint32_t (&w)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]),
                 "=r"(w[7])
               : "l"(ptr));
}

// Barrier over `count` threads (a multiple of 32) of this CTA on named barrier `id`.
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

}  // namespace ptx
}  // namespace b200gemm
