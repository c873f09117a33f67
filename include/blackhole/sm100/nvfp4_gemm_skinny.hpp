#pragma once

// =====================================================================================
// blackhole / sm100 / NVFP4 GEMM, skinny-M schedule (M <= 128: decode-style shapes)
// -------------------------------------------------------------------------------------
// For M <= 128 the GEMM is bound by streaming B (N x K/2 bytes + its scale factors) from
// HBM.  This schedule computes D^T = B . A^T so that 128 rows of B fill the UMMA M = 128
// and the M activation rows become the UMMA N (padded to MPAD = 16/32/64/128; TMA
// zero-fills rows >= M):
//
//   * work unit = (128-row block rb of B, K-slice kt of UnitK = 256 or 512 elements: one or two
//     k-tiles of 128-byte shared-memory rows); U = ceil(N/128) * ceil(K/UnitK) units are
//     split into equal contiguous ranges, one per persistent CTA (stream-K), so every SM
//     streams the same number of bytes;
//   * each CTA walks its range backwards in row-block segments; a segment accumulates in
//     one of two TMEM accumulators (128 lanes x MPAD FP32 columns) so its epilogue overlaps
//     the next segment's loads and MMAs;
//   * a row block that spans several CTAs is finished by the CTA owning its last k-tile:
//     the others (which reach it first) park FP32 partials in the workspace and raise a
//     flag per epilogue warp; the finisher's matching warp adds them in a fixed order
//     (deterministic) and writes BF16.  Only warps exchange data, never whole CTAs, so no
//     CTA-wide barrier sits in the epilogue.
//
// Each CTA parks at most one partial, so the workspace is 8 flags per CTA plus
// grid * MPAD * 128 * 4 bytes of partials (nvfp4_skinny_workspace_bytes).
// A flag is raised by the producer of a partial to its launch's tag and reset to 0 by its
// consumer; the tag is odd and changes with every launch (a generation word next to the ticket
// counter, advanced once per launch), so a flag that a launch left raised because it gave up on
// a bounded wait never matches a later launch's tag: the workspace stays reusable by later
// launches on the same stream (and by graph replays) after an aborted one too.
// Because finishers wait only on lower-numbered CTAs, which were launched no later, the
// dependency never points at a CTA that cannot be resident.
// =====================================================================================

#include <cstdint>

#include <blackhole/sm100/block_scale_format.hpp>
#include <blackhole/sm100/nvfp4_gemm_common.hpp>

namespace blackhole::sm100 {

template <int MPAD_, class Fmt_ = Nvfp4Format, int KpsOverride_ = 0>
struct Nvfp4SkinnyTraits {
  using Fmt = Fmt_;
  using Geo = BlockScaleGeometry<Fmt>;
  static constexpr int SFVecSize = Fmt::SfVec;
  static constexpr int MPAD = MPAD_;            // UMMA N
  static constexpr int TileW = 128;             // rows of B per unit (UMMA M)
  static constexpr int TileK = Fmt::TileK;      // elements per k-tile (128-byte smem rows)
  static constexpr int KSteps = Geo::KSteps;
  static constexpr int RowBytes = Geo::RowBytes;
  // k-tiles per work unit (and shared-memory stage): 2 where B is expanded (MXFP8 x MXFP4,
  // 128-deep k-tiles) and at MPAD = 16 for every format, 1 otherwise.  The per-unit cost
  // (barrier round trip, scale-factor copy and commit issue) is then paid once per 32 KB
  // (4-bit) or 16 KB (expanded) of weights; measured on B200 at N = 28672, K = 8192: M = 16
  // NVFP4 25.5 -> 23.7 us, MXFP4 24.1 -> 21.9 us, MXFP8 x MXFP4 39.0 -> 27.3 us.  Wider
  // activation tiles (MPAD >= 32) keep one k-tile per stage, where the ring depth matters more.
  static constexpr int KPS = KpsOverride_ > 0 ? KpsOverride_ : ((Fmt::BExpand || MPAD <= 16) ? 2 : 1);
  static constexpr int UnitK = KPS * TileK;                 // K-elements per unit
  static constexpr int UnitSteps = KPS * KSteps;            // MMAs per unit
  static constexpr int TileWBytes = TileW * RowBytes;       // one k-tile of B: 16 KB
  static constexpr int TileXBytes = MPAD * RowBytes;        // one k-tile of A: 2..16 KB
  static constexpr int WBytes = KPS * TileWBytes;
  static constexpr int XBytes = KPS * TileXBytes;
  // scale-factor atoms per 128 rows and k-tile: 4 (NVFP4), 2 (MXFP4), 1 (MXFP8 x MXFP4)
  static constexpr int StepsPerAtom = Geo::StepsPerAtom;
  static constexpr int SfAtoms = Geo::SfAtoms;
  static constexpr int UnitAtoms = KPS * SfAtoms;           // scale-factor atoms per unit
  static constexpr int SFBytes = UnitAtoms * 512;           // 2 KB per operand (NVFP4)
  static constexpr int StageBytes = WBytes + XBytes + 2 * SFBytes;
  // global bytes a stage's loads complete (the expanded 4-bit B is half its smem size)
  static constexpr int StageTx = KPS * (TileW * Geo::BRowTx + MPAD * Geo::ARowTx) + 2 * SFBytes;
  // NVFP4 / MXFP4: depths tuned per width.  An expanded 4-bit B (MXFP8 x MXFP4) moves half
  // its shared-memory bytes per stage, so its ring takes every stage that fits (at most 12).
  static constexpr int FitStages =
      (arch_traits<Arch::kSm100>::max_smem_per_cta - 1024 - 8 * (2 * 12 + 5) - 16) / StageBytes;
  static constexpr int Stages = KPS == 2 ? (FitStages < 12 ? FitStages : 12)
                                             : ((MPAD <= 32) ? 9 : (MPAD == 64 ? 8 : 6));
  // units of B prefetched into L2 before the dependency wait (beyond the smem stages): 20
  // k-tiles' worth of weight rows in every format
  static constexpr int L2PrefetchKTiles = 20 / KPS;
  // ranges by ticket: the first CTA to start gets (1 + s) x, the last (1 - s) x the mean
  // work, s = RangeSkew / 64 (measured on B200 at M = 16, N = 28672, K = 8192, back to back,
  // medians of six: skew 6 / 8 / 9 / 10 took 24.14 / 23.78 / 23.75 / 23.92 us, 0 took ~25.5)
  static constexpr int RangeSkew = MPAD <= 16 ? 9 : 6;

  // TMA, MMA, then 4 epilogue warps (one per TMEM sub-partition), or 8 for MPAD >= 64: two per
  // sub-partition, each draining half of the accumulator columns (the last segment's
  // epilogue is on the kernel's critical path; at MPAD = 128 it took ~11 us with 4 warps).
  static constexpr int NumEpiWarps = MPAD >= 64 ? 8 : 4;
  static constexpr int EpiCols = MPAD * 4 / NumEpiWarps;    // accumulator columns per warp
  static constexpr int NumWarps = 2 + NumEpiWarps;
  static constexpr int NumThreads = NumWarps * 32;
  static constexpr int ProducerWarp = 0;
  static constexpr int MmaWarp = 1;
  static constexpr int FirstEpiWarp = 2;

  static constexpr uint32_t TmemCols = 512;
  static constexpr uint32_t AccStride = 128;                // two accumulators: [0,128), [128,256)
  static constexpr uint32_t SfwCol = 256;                   // 4 columns per atom
  static constexpr uint32_t SfxCol = 256 + 4 * UnitAtoms;   // 4 columns per atom

  static constexpr int BarrierBytes = 8 * (2 * Stages + 5) + 16;
  static constexpr int SmemBytes = Stages * StageBytes + BarrierBytes + 1024;
  static_assert(SmemBytes <= arch_traits<Arch::kSm100>::max_smem_per_cta, "smem budget");
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= 128, "UMMA N");
};

// Workspace layout: flag words first, at a fixed place for the device (8 per possible CTA:
// one per epilogue warp, then the ticket counter, padded to 256 bytes), then the FP32
// partials.  Keeping the flags at a fixed offset means a workspace shared by calls of
// different M never sees partial data where a flag should be.
constexpr int kSkinnyFlagsPerCta = 8;
constexpr int64_t nvfp4_skinny_flag_bytes(int num_sms) {
  return (int64_t(num_sms) * 4 * kSkinnyFlagsPerCta + 16 + 255) / 256 * 256;
}
// Bytes of workspace the skinny schedule needs on a device with num_sms SMs at width mpad.
constexpr int64_t nvfp4_skinny_workspace_bytes(int num_sms, int mpad) {
  return nvfp4_skinny_flag_bytes(num_sms) + int64_t(num_sms) * mpad * 128 * 4;
}

inline int nvfp4_skinny_mpad(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

#if defined(__CUDACC__)

struct Nvfp4SkinnyParams {
  CUtensorMap tmap_w;   // B [N][K/2] bytes, box 128 rows x 128 B
  CUtensorMap tmap_x;   // A [M][K/2] bytes, box MPAD rows x 128 B
  const uint8_t* sfw;   // SFB
  const uint8_t* sfx;   // SFA
  uint16_t* d;          // this call's first output column; rows ldd elements apart
  int64_t ldd;
  int num_peers;        // gather mode: further destinations, laid out as d
  uint16_t* peer_d[kMaxGatherPeers];
  float* ws;            // [grid][MPAD][128] partials
  uint32_t* flags;      // [grid][8]: one per epilogue warp
  uint32_t* ticket;     // [0]: entry counter, CTAs take ranges in the order they start;
                        // [1]: launch generation, advanced once per launch
  uint32_t* status;
  uint64_t partial_wait_ns;   // bound of a finisher's wait for a partial (kWaitLimitNs)
  float alpha;
  int M, N, K;
  int kt_per_rb;        // units per 128-row block: ceil(K / UnitK)
  int64_t units;        // ceil(N/128) * ceil(K/UnitK)
  int grid;
  int skew;             // range of ticket t shrinks linearly: density (1 + s - 2 s t / grid), s = skew/64
  int sf_k_atoms;
  int l2_pf;            // k-tiles of B / SFB prefetched into L2 before the previous kernel completes
  int sf_tail;          // K % 256 != 0: scale factors through the atom-granular tensor maps
  CUtensorMap tmap_sfw; // (sf_tail only) SFB [N/128][atoms][512 B], box 4 atoms x 1 block
  CUtensorMap tmap_sfx; // (sf_tail only) SFA [1][atoms][512 B], box 4 atoms
};

namespace skinny_detail {

// First unit of the range of ticket t.  Ranges shrink linearly with the ticket: CTAs that
// start late (on SMs whose previous CTA finished late, or with less time to prefetch before
// the previous kernel completes) get less work.  Monotone, range_start(grid) == units; the
// launcher keeps every range non-empty and the products inside 63 bits.
__device__ __forceinline__ int64_t range_start(const Nvfp4SkinnyParams& p, int t) {
  const int64_t g = p.grid;
  if (p.skew == 0) return int64_t(t) * p.units / g;
  const int64_t num = (64 + p.skew) * int64_t(t) * g - p.skew * int64_t(t) * t;
  return p.units * num / (64 * g * g);
}

// One row-block segment of a CTA's range, visited from the end of the range backwards.
struct Segment {
  int rb, kt0, kt1;
};

struct SegmentWalk {
  int64_t begin, u;
  int KT;
  __device__ __forceinline__ bool next(Segment& s) {
    if (u <= begin) return false;
    const int rb = static_cast<int>((u - 1) / KT);
    const int64_t rb0 = int64_t(rb) * KT;
    const int64_t sb = begin > rb0 ? begin : rb0;
    s.rb = rb;
    s.kt0 = static_cast<int>(sb - rb0);
    s.kt1 = static_cast<int>(u - rb0);
    u = sb;
    return true;
  }
};

__device__ __forceinline__ SegmentWalk walk(const Nvfp4SkinnyParams& p, int c) {
  SegmentWalk w;
  w.begin = range_start(p, c);
  w.u = range_start(p, c + 1);
  w.KT = p.kt_per_rb;
  return w;
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

}  // namespace skinny_detail

template <class KT, bool kGather = false>
__global__ void __launch_bounds__(KT::NumThreads, 1)
    nvfp4_gemm_skinny_kernel(const __grid_constant__ Nvfp4SkinnyParams p) {
#if defined(BLACKHOLE_ARCH_SM100)
  using namespace ptx;
  using namespace skinny_detail;
  constexpr int S = KT::Stages;
  constexpr int MPAD = KT::MPAD;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw);
  auto st_w = [&](int s) { return base + uint32_t(s) * KT::StageBytes; };
  auto st_x = [&](int s) { return st_w(s) + KT::WBytes; };
  auto st_sfw = [&](int s) { return st_x(s) + KT::XBytes; };
  auto st_sfx = [&](int s) { return st_sfw(s) + KT::SFBytes; };
  const uint32_t bars = base + S * KT::StageBytes;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
  auto acc_full = [&](int a) { return bars + 8u * (2 * S + a); };
  auto acc_empty = [&](int a) { return bars + 8u * (2 * S + 2 + a); };
  const uint32_t drain_bar = bars + 8u * (2 * S + 4);
  uint32_t* const tmem_slot =
      reinterpret_cast<uint32_t*>(base_ptr + (bars - base) + 8 * (2 * S + 5));
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  volatile uint32_t* const ticket_slot = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);
  volatile uint32_t* const gen_slot = reinterpret_cast<volatile uint32_t*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // Ranges go to CTAs in the order they start.  The taker of the last ticket resets the
    // counter for the next launch; that launch starts taking tickets only after every CTA of
    // this one has passed pdl_launch_dependents below, i.e. after the reset.
    // The generation is read before the ticket is taken and advanced by the last taker after
    // its reset, so every CTA of a launch reads the same value (the fences order the read, the
    // ticket and the advance) and the next launch reads the advanced one.
    const uint32_t gen = ld_acquire(p.ticket + 1);
    __threadfence();
    const uint32_t t = atomicAdd(p.ticket, 1u);
    if (t == uint32_t(p.grid) - 1u) {
      atomicExch(p.ticket, 0u);
      __threadfence();
      atomicExch(p.ticket + 1, gen + 1u);
      __threadfence();
    }
    *ticket_slot = t;
    *gen_slot = (gen << 1) | 1u;
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(acc_full(a), 1);
      mbar_init(acc_empty(a), KT::NumEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == KT::MmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), KT::TmemCols);
    tmem_relinquish();
  }
  if (warp == KT::ProducerWarp && lane == 0) {
    prefetch_tmap(&p.tmap_w);
    prefetch_tmap(&p.tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int c = static_cast<int>(*ticket_slot);
  const uint32_t tag = *gen_slot;   // this launch's flag value (odd, never 0)
  pdl_launch_dependents();  // the next kernel may claim SMs as ours exit
  // The previous kernel in the stream must be complete before any operand or the workspace is
  // read or written; the producer first issues L2 prefetches of B / SFB.
  if (warp != KT::ProducerWarp) pdl_wait_prior_grid();

  if (warp == KT::ProducerWarp) {
    // ------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();   // B is streamed exactly once
      const uint64_t pol_x = l2_policy_evict_last();    // A is re-read by every CTA
      // Before the previous kernel in the stream has completed, only L2 prefetches of this
      // CTA's first l2_pf k-tiles of B / SFB are issued: HBM keeps streaming across the kernel
      // boundary, and since L2 is the point of coherence a prefetch can never make a later
      // load see stale data, whatever the previous kernel writes.
      // L2 prefetch of this CTA's first l2_pf weight tiles, before the wait.  (Continuing the
      // stream in steady state, one prefetch per unit loaded, measured ~5 us slower per launch:
      // every extra copy-engine request costs more than the depth it adds.)
      SegmentWalk wa = walk(p, c);
      Segment sa;
      int kta = 0, kta_end = 0;
      auto prefetch_next = [&]() {
        if (kta == kta_end) {
          if (!wa.next(sa)) return;
          kta = sa.kt0;
          kta_end = sa.kt1;
        }
        const int kt = kta++;
#pragma unroll
        for (int h = 0; h < KT::KPS; ++h)   // (a K tail's last unit may end inside its first half)
          if ((kt * KT::KPS + h) * KT::TileK < p.K)
            tma_prefetch_l2_2d(&p.tmap_w, (kt * KT::KPS + h) * KT::RowBytes, sa.rb * KT::TileW);
        // only the atoms that exist (the last unit of a K tail has fewer)
        const int atoms = min(KT::UnitAtoms, p.sf_k_atoms - KT::UnitAtoms * kt);
        if (atoms > 0)
          bulk_prefetch_l2(p.sfw + int64_t(sa.rb) * p.sf_k_atoms * 512 + int64_t(kt) * KT::UnitAtoms * 512,
                           uint32_t(atoms) * 512u);
      };
      for (int i = 0; i < p.l2_pf; ++i) prefetch_next();
      pdl_wait_prior_grid();
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      SegmentWalk w = walk(p, c);
      Segment sg;
      while (ok && w.next(sg)) {
        const uint8_t* sfw_rb = p.sfw + int64_t(sg.rb) * p.sf_k_atoms * 512;
        for (int kt = sg.kt0; kt < sg.kt1; ++kt) {
          if (!wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.status, kStatusLoadTimeout)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          const int64_t k_off = int64_t(kt) * KT::UnitAtoms * 512;
          mbar_arrive_expect_tx(fb, KT::StageTx);
          // A (small, L2-resident) ahead of B in the copy engine's queue; a unit's k-tiles sit
          // side by side in the stage (rows past K read zeros)
#pragma unroll
          for (int h = 0; h < KT::KPS; ++h)
            tma_load_2d(st_x(stage) + h * KT::TileXBytes, &p.tmap_x, fb,
                        (kt * KT::KPS + h) * KT::RowBytes, 0, pol_x);
          if (p.sf_tail)  // atoms past K read zeros
            tma_load_3d(st_sfx(stage), &p.tmap_sfx, fb, 0, KT::UnitAtoms * kt, 0, pol_x);
          else
            bulk_load(st_sfx(stage), p.sfx + k_off, KT::SFBytes, fb, pol_x);
#pragma unroll
          for (int h = 0; h < KT::KPS; ++h)
            tma_load_2d(st_w(stage) + h * KT::TileWBytes, &p.tmap_w, fb,
                        (kt * KT::KPS + h) * KT::RowBytes, sg.rb * KT::TileW, pol_w);
          if (p.sf_tail)
            tma_load_3d(st_sfw(stage), &p.tmap_sfw, fb, 0, KT::UnitAtoms * kt, sg.rb, pol_w);
          else
            bulk_load(st_sfw(stage), sfw_rb + k_off, KT::SFBytes, fb, pol_w);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < S; ++s) {
          if (issued > s) {
            const int64_t cnt = (issued - 1 - s) / S + 1;
            detail::drain_wait(full_bar(s), uint32_t((cnt - 1) & 1));
          }
        }
      }
    }
  } else if (warp == KT::MmaWarp) {
    // ------------------------------ MMA issuer --------------------------------------
    // swap-AB: the MMA's A operand is the weights (B), its B operand the activations (A)
    constexpr uint32_t idesc = idesc_block_scaled(128, MPAD, KT::Fmt::BFormat, KT::Fmt::AFormat,
                                                  KT::Fmt::ScaleType);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true, issued_any = false;
    SegmentWalk w = walk(p, c);
    Segment sg;
    while (ok && w.next(sg)) {
      if (!wait_bounded_warp(acc_empty(acc), acc_phase ^ 1u, abort_flag, p.status, kStatusMmaTimeout)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem + KT::AccStride * acc;
      if (!wait_bounded_warp(full_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kt = sg.kt0; kt < sg.kt1; ++kt) {
        const int nstage = stage + 1 == S ? 0 : stage + 1;
        const uint32_t nphase = stage + 1 == S ? (phase ^ 1u) : phase;
        const bool more = kt + 1 < sg.kt1;
        const uint32_t ready = more ? mbar_probe(full_bar(nstage), nphase) : 1u;
        {
#pragma unroll
          for (int j = 0; j < KT::UnitAtoms; ++j) {
            tc_cp_32x128b_warpx4_w(tmem + KT::SfwCol + 4 * j, desc_sf_atom(st_sfw(stage) + 512 * j));
            tc_cp_32x128b_warpx4_w(tmem + KT::SfxCol + 4 * j, desc_sf_atom(st_sfx(stage) + 512 * j));
          }
#pragma unroll
          for (int j = 0; j < KT::UnitSteps; ++j) {
            // k-tile h of the unit, k-step jj inside its swizzled rows (+32 bytes per step)
            const int h = j / KT::KSteps, jj = j % KT::KSteps;
            const uint64_t wdesc = desc_kmajor_sw128(st_w(stage) + h * KT::TileWBytes);
            const uint64_t xdesc = desc_kmajor_sw128(st_x(stage) + h * KT::TileXBytes);
            const int at = j / KT::StepsPerAtom;
            const uint32_t sid = KT::Geo::sf_id(j);   // byte in the entry
            tc_mma_bs_w<typename KT::Fmt>(
                d_tmem, wdesc + 2 * jj, xdesc + 2 * jj, idesc_with_sf_id(idesc, sid),
                sf_tmem_addr(tmem + KT::SfwCol + 4 * at, sid),
                sf_tmem_addr(tmem + KT::SfxCol + 4 * at, sid), (kt != sg.kt0 || j != 0) ? 1u : 0u);
          }
          tc_commit_w(empty_bar(stage));
          issued_any = true;
        }
        stage = nstage;
        phase = nphase;
        if (more) {
          if (!__all_sync(0xFFFFFFFFu, ready != 0u) &&
              !wait_bounded_warp(full_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
      }
      if (!ok) break;
      tc_commit_w(acc_full(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (!ok && issued_any) {
      tc_commit_w(drain_bar);
      detail::drain_wait(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ----------------------------------------
    constexpr int EC = KT::EpiCols;
    const int q = warp & 3;                                       // TMEM sub-partition
    const int m0 = ((warp - KT::FirstEpiWarp) >> 2) * EC;        // first column (row of D)
    const int fi = q + 4 * ((warp - KT::FirstEpiWarp) >> 2);     // this warp's flag slot
    const int n_local = 32 * q + lane;                            // row of the B block
    // Adds the FP32 partials parked by the earlier CTAs sharing row block sg.rb (in a fixed
    // order: deterministic) into v; false if a bounded wait gave up.
    auto add_partials = [&](const Segment& sg, float (&v)[EC]) -> bool {
      const int64_t rb0 = int64_t(sg.rb) * p.kt_per_rb;
      for (int cc = c - 1; cc >= 0 && range_start(p, cc + 1) > rb0; --cc) {
        uint32_t* flag = p.flags + kSkinnyFlagsPerCta * cc + fi;
        int ready = 1;
        if (lane == 0) {
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire(flag) != tag) {
            if (*abort_flag) { ready = 0; break; }
            if (globaltimer_ns() - t0 > p.partial_wait_ns) {
              *abort_flag = 1;
              if (p.status) atomicOr(p.status, kStatusEpilogueTimeout);
              ready = 0;
              break;
            }
          }
        }
        ready = __shfl_sync(0xFFFFFFFFu, ready, 0);
        if (!ready) return false;
        (void)ld_acquire(flag);
        const float* src = p.ws + (int64_t(cc) * MPAD + m0) * 128 + n_local;
#pragma unroll
        for (int m = 0; m < EC; ++m)
          if (m0 + m < p.M) v[m] += __ldcg(src + m * 128);
        __syncwarp();
        if (lane == 0) st_release(flag, 0u);
      }
      return true;
    };
    // When a warp drains at most 32 columns, the partials of a finished row block are
    // fetched before its accumulator is ready, so that their latency is off the critical path.
    constexpr bool kEarlyPartials = EC <= 32;
    int acc = 0;
    uint32_t acc_phase = 0;
    SegmentWalk w = walk(p, c);
    Segment sg;
    while (w.next(sg)) {
      const bool finisher = sg.kt1 == p.kt_per_rb;
      float part[kEarlyPartials ? EC : 1];
      if constexpr (kEarlyPartials) {
#pragma unroll
        for (int m = 0; m < EC; ++m) part[m] = 0.f;
        if (finisher && sg.kt0 > 0 && !add_partials(sg, part)) break;
      }
      if (!wait_bounded_warp(acc_full(acc), acc_phase, abort_flag, p.status, kStatusEpilogueTimeout))
        break;
      tc_fence_after();
      float v[EC];
      {
        const uint32_t t =
            tmem + (static_cast<uint32_t>(32 * q) << 16) + KT::AccStride * acc + uint32_t(m0);
#pragma unroll
        for (int j = 0; j < EC / 16; ++j) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t + 16 * j, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            asm volatile("" : "+r"(r[i]));
            v[16 * j + i] = __uint_as_float(r[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }

      const int n = sg.rb * 128 + n_local;
      if (!finisher) {
        // Partial of a row block finished by a later CTA: park it, then raise this warp's flag.
        float* dst = p.ws + (int64_t(c) * MPAD + m0) * 128 + n_local;
#pragma unroll
        for (int m = 0; m < EC; ++m)
          if (m0 + m < p.M) __stcg(dst + m * 128, v[m]);
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release(p.flags + kSkinnyFlagsPerCta * c + fi, tag);
        continue;
      }
      if constexpr (kEarlyPartials) {
#pragma unroll
        for (int m = 0; m < EC; ++m) v[m] += part[m];
      } else {
        if (sg.kt0 > 0 && !add_partials(sg, v)) break;
      }
      const float a = p.alpha;
#pragma unroll
      for (int m = 0; m < EC; ++m) {
        if (m0 + m < p.M && n < p.N) {
          __nv_bfloat16 b = __float2bfloat16_rn(a * v[m]);
          const uint16_t bits = *reinterpret_cast<uint16_t*>(&b);
          // the plain GEMM keeps D's own row stride; gather mode (its own instantiation, so
          // the plain one carries none of its code) also stores to every further buffer
          const int64_t off = int64_t(m0 + m) * (kGather ? p.ldd : int64_t(p.N)) + n;
          p.d[off] = bits;
          if constexpr (kGather)
            for (int q = 0; q < p.num_peers; ++q) p.peer_d[q][off] = bits;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == KT::MmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, KT::TmemCols);
  }
#endif  // BLACKHOLE_ARCH_SM100
}

namespace detail {

template <class KT>
inline cudaError_t launch_skinny(int M, int N, int K, const void* A, const void* SFA, const void* B,
                                 const void* SFB, void* D, float alpha, void* ws, int64_t ws_bytes,
                                 int grid_cap, bool prefetch, DeviceState* st, cudaStream_t stream,
                                 int l2_prefetch_ktiles = KT::L2PrefetchKTiles,
                                 int skew = KT::RangeSkew, const GatherSpec* g = nullptr,
                                 uint64_t partial_wait_ns = ptx::kWaitLimitNs) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // gather mode has its own instantiation (NVFP4 only: the gather entry point's format)
  constexpr bool kCanGather = std::is_same_v<typename KT::Fmt, Nvfp4Format>;
  if (g && !kCanGather) return cudaErrorInvalidValue;
  auto* kernel = nvfp4_gemm_skinny_kernel<KT, false>;
  if constexpr (kCanGather)
    if (g) kernel = nvfp4_gemm_skinny_kernel<KT, true>;
  e = set_smem_once(kernel, KT::SmemBytes, dev);
  if (e != cudaSuccess) return e;
  Nvfp4SkinnyParams p;
  e = make_b_tmap<typename KT::Fmt>(&p.tmap_w, B, N, K, 128);
  if (e != cudaSuccess) return e;
  e = make_a_tmap<typename KT::Fmt>(&p.tmap_x, A, M, K, KT::MPAD);
  if (e != cudaSuccess) return e;
  p.kt_per_rb = (K + KT::UnitK - 1) / KT::UnitK;
  p.sf_tail = K % KT::UnitK != 0;
  if (p.sf_tail) {
    e = make_sf_tmap_atoms(&p.tmap_sfw, SFB, N, K, 1, KT::UnitAtoms, KT::SFVecSize);
    if (e != cudaSuccess) return e;
    e = make_sf_tmap_atoms(&p.tmap_sfx, SFA, M, K, 1, KT::UnitAtoms, KT::SFVecSize);
    if (e != cudaSuccess) return e;
  }
  p.units = int64_t((N + 127) / 128) * p.kt_per_rb;
  int grid = grid_cap < st->num_sms ? grid_cap : st->num_sms;
  if (p.units < grid) grid = static_cast<int>(p.units);
  if (nvfp4_skinny_workspace_bytes(st->num_sms, KT::MPAD) > ws_bytes) return cudaErrorInvalidValue;
  p.sfw = static_cast<const uint8_t*>(SFB);
  p.sfx = static_cast<const uint8_t*>(SFA);
  p.d = static_cast<uint16_t*>(D);
  p.ldd = N;
  p.num_peers = 0;
  if (g) {
    p.d = static_cast<uint16_t*>(g->dst[0]) + g->col0;
    p.ldd = g->ldd;
    p.num_peers = g->ndst - 1;
  }
  for (int i = 0; i < kMaxGatherPeers; ++i)
    p.peer_d[i] = g && i + 1 < g->ndst ? static_cast<uint16_t*>(g->dst[i + 1]) + g->col0 : nullptr;
  p.flags = static_cast<uint32_t*>(ws);
  p.ticket = p.flags + kSkinnyFlagsPerCta * st->num_sms;
  p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + nvfp4_skinny_flag_bytes(st->num_sms));
  p.status = st->status;
  p.partial_wait_ns = partial_wait_ns;
  p.alpha = alpha;
  p.M = M;
  p.N = N;
  p.K = K;
  p.grid = grid;
  // skew only where every range keeps >= 2 units and range_start cannot overflow
  p.skew = (skew > 0 && skew < 64 && p.units * (64 - skew) >= int64_t(2) * 64 * grid &&
            p.units < (int64_t(1) << 62) / (128 * int64_t(grid) * grid))
               ? skew
               : 0;
  p.sf_k_atoms = static_cast<int>(sf_k_atoms_vs(K, KT::SFVecSize));
  p.l2_pf = prefetch ? l2_prefetch_ktiles : 0;
  e = launch_pdl(kernel, dim3(grid), dim3(KT::NumThreads), KT::SmemBytes,
                 stream, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace detail

// Skinny-M GEMM with a caller-provided workspace of at least
// nvfp4_skinny_workspace_bytes(num_SMs, nvfp4_skinny_mpad(M)) bytes, zero-filled before its
// first use; every launch, one that gave up on a bounded wait included, leaves it usable by
// the next launch on the stream.  M in [1, 128].
//
// With prefetch the kernel, launched as a programmatic dependent of the previous kernel in
// the stream, issues L2 prefetches of the first B / SFB tiles of its range while that kernel
// is finishing; every load, store and workspace access still waits for its completion, so
// the results are those of plain stream order either way.
template <class Fmt = Nvfp4Format>
inline cudaError_t block_scaled_bf16_gemm_skinny(int M, int N, int K, void const* A,
                                                 void const* SFA, void const* B, void const* SFB,
                                                 void* D, float alpha, void* workspace,
                                                 int64_t workspace_bytes,
                                                 cudaStream_t stream = nullptr,
                                                 int grid_cap = 1 << 30, bool prefetch = true,
                                                 const detail::GatherSpec* g = nullptr,
                                                 uint64_t partial_wait_ns = ptx::kWaitLimitNs) {
  cudaError_t e = nvfp4_check_args(M, N, K, A, SFA, B, SFB, D);
  if (e != cudaSuccess) return e;
  e = detail::format_check_args<Fmt>(K, B);
  if (e != cudaSuccess) return e;
  if (M > 128 || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 15u))
    return cudaErrorInvalidValue;
  detail::DeviceState* st = detail::prepare_device();
  if (!st) return cudaErrorInvalidDevice;
  if (st->init_err != cudaSuccess) return st->init_err;
  switch (nvfp4_skinny_mpad(M)) {
    case 16:
      return detail::launch_skinny<Nvfp4SkinnyTraits<16, Fmt>>(
          M, N, K, A, SFA, B, SFB, D, alpha, workspace, workspace_bytes, grid_cap, prefetch, st, stream,
          Nvfp4SkinnyTraits<16, Fmt>::L2PrefetchKTiles, Nvfp4SkinnyTraits<16, Fmt>::RangeSkew, g,
          partial_wait_ns);
    case 32:
      return detail::launch_skinny<Nvfp4SkinnyTraits<32, Fmt>>(
          M, N, K, A, SFA, B, SFB, D, alpha, workspace, workspace_bytes, grid_cap, prefetch, st, stream,
          Nvfp4SkinnyTraits<32, Fmt>::L2PrefetchKTiles, Nvfp4SkinnyTraits<32, Fmt>::RangeSkew, g,
          partial_wait_ns);
    case 64:
      return detail::launch_skinny<Nvfp4SkinnyTraits<64, Fmt>>(
          M, N, K, A, SFA, B, SFB, D, alpha, workspace, workspace_bytes, grid_cap, prefetch, st, stream,
          Nvfp4SkinnyTraits<64, Fmt>::L2PrefetchKTiles, Nvfp4SkinnyTraits<64, Fmt>::RangeSkew, g,
          partial_wait_ns);
    default:
      return detail::launch_skinny<Nvfp4SkinnyTraits<128, Fmt>>(
          M, N, K, A, SFA, B, SFB, D, alpha, workspace, workspace_bytes, grid_cap, prefetch, st, stream,
          Nvfp4SkinnyTraits<128, Fmt>::L2PrefetchKTiles, Nvfp4SkinnyTraits<128, Fmt>::RangeSkew, g,
          partial_wait_ns);
  }
}

// The NVFP4 operator's skinny schedule (the reference's format).
inline cudaError_t nvfp4_bf16_gemm_skinny(int M, int N, int K, void const* A, void const* SFA,
                                          void const* B, void const* SFB, void* D, float alpha,
                                          void* workspace, int64_t workspace_bytes,
                                          cudaStream_t stream = nullptr, int grid_cap = 1 << 30,
                                          bool prefetch = true) {
  return block_scaled_bf16_gemm_skinny<Nvfp4Format>(M, N, K, A, SFA, B, SFB, D, alpha, workspace,
                                                    workspace_bytes, stream, grid_cap, prefetch);
}

#endif  // __CUDACC__

}  // namespace blackhole::sm100
