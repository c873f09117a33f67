#pragma once

// Thin inline-PTX wrappers for the sm_100a datapath used by the NVFP4 kernels:
// mbarriers, TMA tensor and bulk copies, TMEM allocation, tcgen05 copy / MMA / commit /
// load.  Every wait on an mbarrier is bounded (see wait_bounded): a pipeline that stops
// making progress records an error code and the kernel returns instead of hanging.

#include <cstdint>

#include <blackhole/sm100/block_scale_format.hpp>

#if defined(__CUDACC__)
#include <cuda.h>  // CUtensorMap

namespace blackhole::sm100::ptx {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- programmatic dependent launch ---------------------------------------------------------
// Both are no-ops unless the kernel was launched with programmatic stream serialization.
// launch_dependents lets the next kernel in the stream be scheduled (its CTAs take SMs as
// this kernel's CTAs exit); wait blocks until the previous kernel has completed and its
// memory is visible, so it goes before the first read of inputs or write of outputs.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- mbarrier ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// A wait gives up after this long: every legitimate wait in these kernels lasts
// microseconds (one k-tile of TMA or one tile of MMAs).
constexpr uint64_t kWaitLimitNs = 4000000000ull;

// Non-blocking-use probe: issue it early and test the result later; the barrier latency then
// hides behind whatever the warp issues in between (measured on B200: an MMA warp that
// probes the next stage before issuing the current k-tile keeps the tensor pipe at 100%,
// against ~78% when it waits for the next stage after the MMAs).
__device__ __forceinline__ uint32_t mbar_probe(uint32_t bar, uint32_t parity) {
  return mbar_try_wait(bar, parity) ? 1u : 0u;
}

// Waits for the phase with the given parity to complete.  Returns false when the CTA's
// abort flag is raised (another role gave up) or when the time limit passes; in that case
// the flag is raised and `code` is or-ed into *status so the host can see it.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity,
                                             volatile int* abort_flag, uint32_t* status,
                                             uint32_t code, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        if (status) atomicOr(status, code);
        return false;
      }
    }
  }
}

// Warp-uniform form for waits that all 32 lanes of a warp execute: every lane returns the
// same answer (completion is agreed with __all_sync, giving up is lane 0's decision), so a
// warp never splits between "done" and "abort" and no later warp-wide operation can hang.
__device__ __forceinline__ bool wait_bounded_warp(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, uint32_t* status,
                                                  uint32_t code,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (__all_sync(0xFFFFFFFFu, mbar_try_wait(bar, parity))) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (__all_sync(0xFFFFFFFFu, mbar_try_wait(bar, parity))) return true;
    if ((i & 63u) == 0) {
      int give_up = 0;
      if ((threadIdx.x & 31) == 0) {
        if (*abort_flag) {
          give_up = 1;
        } else if (globaltimer_ns() - t0 > limit_ns) {
          *abort_flag = 1;
          if (status) atomicOr(status, code);
          give_up = 1;
        }
      }
      if (__shfl_sync(0xFFFFFFFFu, give_up, 0)) return false;
    }
  }
}

// ---- TMA / bulk copies -------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory; completes `bytes` on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Contiguous global -> shared bulk copy (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// Prefetch into L2 only (no shared memory, no barrier): a 2-D tile of a tensor map, or a
// contiguous byte range (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* m, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- TMEM --------------------------------------------------------------------------------
// Whole-warp operations.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Copies a 512-byte scale-factor atom (32 rows x 16 bytes) from shared memory into 4 TMEM
// columns, replicated into all four 32-lane sub-partitions.
__device__ __forceinline__ void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// D(tmem) (+)= A(smem) . B(smem)^T with per-16 UE4M3 scale factors read from TMEM.
__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread (thread i = lane i).
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
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Makes later uses of r[] depend on code placed after tmem_ld_wait().
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

// ---- warp-wide issue forms ------------------------------------------------------------------
// The MMA warp computes every operand (descriptors, TMEM addresses) with all 32 lanes, so
// the values are warp-uniform, and each tcgen05 instruction is issued by the lane that
// elect.sync picks inside the asm.  Measured on B200: a k-tile of 12 scale-factor copies +
// 4 MMAs (128x256x64) issues in 513 clocks this way, i.e. at the MMA rate, against 914
// clocks when lane 0 alone computes and issues.  All 32 lanes must call these together; the
// same lane is elected every time, so commits track that lane's MMAs.
__device__ __forceinline__ void tc_cp_32x128b_warpx4_w(uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\t"
      "@P tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc)
      : "memory");
}
// SfVec = 16: scale blocks of 16 elements (NVFP4); 32: blocks of 32 (MXFP4).
template <int SfVec = 16>
__device__ __forceinline__ void tc_mma_nvf4_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                              uint32_t accumulate) {
  static_assert(SfVec == 16 || SfVec == 32, "scale block");
  if constexpr (SfVec == 16) {
    asm volatile(
        "{\n\t.reg .pred p, P;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "@P tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
        "}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, P;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "@P tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
        "}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  }
}
// kind::mxf8f6f4 (one UE8M0 scale per 32 elements, the instruction's only block size).
__device__ __forceinline__ void tc_mma_f8f6f4_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, P;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "@P tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// The block-scaled MMA of a format (block_scale_format.hpp), one CTA.
template <class Fmt>
__device__ __forceinline__ void tc_mma_bs_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                            uint32_t accumulate) {
  if constexpr (Fmt::Kind == MmaKind::kMxf8f6f4)
    tc_mma_f8f6f4_w(d_tmem, adesc, bdesc, idesc, sfa_tmem, sfb_tmem, accumulate);
  else
    tc_mma_nvf4_w<Fmt::SfVec>(d_tmem, adesc, bdesc, idesc, sfa_tmem, sfb_tmem, accumulate);
}
__device__ __forceinline__ void tc_commit_w(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\t"
      "@P tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_cp_32x128b_warpx4_pair_w(uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\t"
      "@P tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc)
      : "memory");
}
template <int SfVec = 16>
__device__ __forceinline__ void tc_mma_nvf4_pair_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                   uint32_t idesc, uint32_t sfa_tmem,
                                                   uint32_t sfb_tmem, uint32_t accumulate) {
  static_assert(SfVec == 16 || SfVec == 32, "scale block");
  if constexpr (SfVec == 16) {
    asm volatile(
        "{\n\t.reg .pred p, P;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "@P tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
        "}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, P;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "@P tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
        "}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  }
}
__device__ __forceinline__ void tc_mma_f8f6f4_pair_w(uint32_t d_tmem, uint64_t adesc,
                                                     uint64_t bdesc, uint32_t idesc,
                                                     uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, P;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "@P tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
template <class Fmt>
__device__ __forceinline__ void tc_mma_bs_pair_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t sfa_tmem,
                                                 uint32_t sfb_tmem, uint32_t accumulate) {
  if constexpr (Fmt::Kind == MmaKind::kMxf8f6f4)
    tc_mma_f8f6f4_pair_w(d_tmem, adesc, bdesc, idesc, sfa_tmem, sfb_tmem, accumulate);
  else
    tc_mma_nvf4_pair_w<Fmt::SfVec>(d_tmem, adesc, bdesc, idesc, sfa_tmem, sfb_tmem, accumulate);
}
__device__ __forceinline__ void tc_commit_pair_w(uint32_t cluster_bar) {
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\t"
      "@P tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          cluster_bar)
      : "memory");
}

// ---- clusters and the 2-SM (cta_group::2) datapath ---------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Arrive on an mbarrier of any CTA in the cluster (shared::cluster address).
// The arrival has release semantics at CTA scope only: what it publishes to the other CTA
// is tensor-memory state, ordered by the tcgen05.fence pair around the barrier, not generic
// memory.  (A cluster-scope release also waits for this thread's earlier memory traffic to
// become visible cluster-wide: measured ~2k clocks per tile in the epilogue on B200.)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of the pair's leader CTA (cluster address `leader_bar`).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m,
                                                 uint32_t leader_bar, int32_t x, int32_t y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(leader_bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// 3-D tiled TMA load into this CTA's shared memory (x innermost); completes on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int32_t x, int32_t y, int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}
// 3-D form of tma_load_2d_pair (x innermost).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* m,
                                                 uint32_t leader_bar, int32_t x, int32_t y,
                                                 int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(leader_bar), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Arrive on `cluster_bar` (any CTA of the pair) when the pair's MMAs issued so far are done.
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_bar)
               : "memory");
}
// Scale-factor atom copy into both CTAs of the pair (each from its own shared memory).
__device__ __forceinline__ void tc_cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
// 256 x N x 64 block-scaled MMA over the CTA pair (issued by the leader only).
__device__ __forceinline__ void tc_mma_nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t sfa_tmem,
                                                 uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// ---- TMA stores ----------------------------------------------------------------------------
// 2-D tiled TMA store from this CTA's shared memory (bulk-group completion).  Coordinates
// must be non-negative; the part of the box outside the tensor is not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, uint32_t src, int32_t x,
                                             int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ---- shared-memory matrix descriptors (tcgen05 format, version 1) -----------------------
// K-major operand tile stored as ROW_BYTES-byte rows with the matching swizzle (as TMA writes
// it with CU_TENSOR_MAP_SWIZZLE_128B / _64B / _32B); 8-row groups are 8 * ROW_BYTES apart.
template <int ROW_BYTES>
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  static_assert(ROW_BYTES == 128 || ROW_BYTES == 64 || ROW_BYTES == 32, "swizzle width");
  constexpr uint64_t layout = ROW_BYTES == 128 ? 2 : (ROW_BYTES == 64 ? 4 : 6);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address, 16-byte units
  d |= static_cast<uint64_t>(1) << 16;                 // leading byte offset (unused here)
  d |= static_cast<uint64_t>((8 * ROW_BYTES) >> 4) << 32;  // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1) << 46;                 // descriptor version (sm_100)
  d |= layout << 61;                                   // swizzle mode
  return d;
}
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) { return desc_kmajor<128>(saddr); }
// Unswizzled 32-row x 16-byte block (a scale-factor atom): 8-row core matrices 128 B apart.
__device__ __forceinline__ uint64_t desc_sf_atom(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}

// Block-scaled instruction descriptor: element formats of the MMA's A and B operands (bits 7-9,
// 10-12; kind::mxf4nvf4 E2M1 = 1, kind::mxf8f6f4 E4M3 = 0 / E2M1 = 5), scale format (bit 23),
// N >> 3 (bits 17-22), M >> 4 (bits 24-28); both operands K-major.
__host__ __device__ constexpr uint32_t idesc_block_scaled(int m, int n, uint32_t a_fmt,
                                                          uint32_t b_fmt, uint32_t scale_type) {
  return (a_fmt << 7) | (b_fmt << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (scale_type << 23) | (static_cast<uint32_t>(m >> 4) << 24);
}
// Scale-factor byte ID of both operands (bits 29-30 for A, 4-5 for B): which byte of each
// 32-bit scale-factor column an MMA starts at.  An atom holds 4 bytes per row: with
// 32-element blocks it serves two 64-deep kind::mxf4nvf4 MMAs (IDs 0 and 2) or four 32-deep
// kind::mxf8f6f4 MMAs (IDs 0..3); with 16-element blocks one MMA reads all 4 (ID 0).
__host__ __device__ constexpr uint32_t idesc_with_sf_id(uint32_t idesc, uint32_t id) {
  return idesc | (id << 29) | (id << 4);
}
// The same ID is also put in bits 30-31 of the scale-factor TMEM address operands, the form
// CUTLASS's UMMA atoms use (the lane field of these addresses is 0).  Measured on B200: the
// MMA takes the ID from the descriptor; with the ID only in the address every MMA read byte 0.
__host__ __device__ constexpr uint32_t sf_tmem_addr(uint32_t taddr, uint32_t id) {
  return taddr | (id << 30);
}

__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

}  // namespace blackhole::sm100::ptx

#endif  // __CUDACC__
