#pragma once

// =====================================================================================
// blackhole / sm100 / NVFP4 GEMM, two-SM schedule (cta_group::2, 256 x 256 tiles)
// -------------------------------------------------------------------------------------
// A cluster of two CTAs (one TPC) computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 64 per instruction):
//
//   * CTA r of the pair loads rows [128r, 128r+128) of the A tile and of the B tile, its
//     own 128 rows of SFA and all 256 rows of SFB (TMA, 128B swizzle for A/B) into a
//     5-stage ring of 38 KB stages.  Every load of either CTA completes on a barrier of the
//     leader CTA (TMA .cta_group::2) that expects the bytes of both CTAs: "full" for A / B,
//     and for NVFP4 a separate scale-factor barrier per stage (its loads are issued first).
//   * The leader copies both CTAs' scale factors to their TMEM (tcgen05.cp.cta_group::2;
//     for NVFP4 split between a copy warp and the MMA warp, see the traits), and its MMA
//     warp issues the MMAs, which read A/B halves from both CTAs'
//     shared memory and write each CTA's 128 x 256 FP32 accumulator into its own TMEM.
//     Its commits arrive on the "empty" barriers of both CTAs and, per tile, on both CTAs'
//     "acc_full" barriers.
//   * Each CTA's 8 epilogue warps drain its own accumulator, arrive on the leader's
//     "acc_empty" barrier and write alpha * acc as BF16 through a 128B-swizzled 4 KB
//     shared-memory box per warp and a TMA tensor store (full-line, coalesced writes; the
//     store clips rows / columns past the edge of D).
//
// Per SM and per 128-clock MMA this moves 38 KB into shared memory instead of the 54 KB a
// one-SM 128 x 256 tile needs, and B crosses L2 -> SM once per pair instead of twice.
// Scale factors are fetched through 3-D tensor maps ([row block][k-tile][2 KB]) as whole 2 KB
// rows, one request per operand and k-tile (ragged M / N edges read zeros): on B200 every
// scale-factor request in flight slows the tensor pipe far beyond its bytes (as four 512-byte
// rows per block they cost ~20% of the mainloop; as 2 KB rows ~10%).
// =====================================================================================

#include <blackhole/sm100/block_scale_format.hpp>
#include <blackhole/sm100/nvfp4_gemm_common.hpp>

namespace blackhole::sm100 {

template <int Stages_ = 5, class Fmt_ = Nvfp4Format, bool OverlapAcc_ = false>
struct Nvfp4Gemm2SmTraitsT {
  using Fmt = Fmt_;
  using Geo = BlockScaleGeometry<Fmt>;
  static constexpr int SFVecSize = Fmt::SfVec;
  static constexpr int TileM = 256;              // per pair (UMMA M)
  static constexpr int CtaM = 128;
  static constexpr int TileN = 256;              // UMMA N
  static constexpr int CtaN = 128;               // B rows held per CTA
  static constexpr int TileK = Fmt::TileK;       // elements per k-tile (128-byte smem rows)
  static constexpr int KSteps = Geo::KSteps;
  static constexpr int Stages = Stages_;

  static constexpr int RowBytes = Geo::RowBytes;
  static constexpr int ABytes = CtaM * RowBytes;           // 16 KB
  static constexpr int BBytes = CtaN * RowBytes;           // 16 KB
  static constexpr int ATx = CtaM * Geo::ARowTx;           // global bytes per k-tile
  static constexpr int BTx = CtaN * Geo::BRowTx;
  // scale-factor atoms per 128 rows and k-tile: 4 (NVFP4), 2 (MXFP4), 1 (MXFP8 x MXFP4)
  static constexpr int StepsPerAtom = Geo::StepsPerAtom;
  static constexpr int SfAtoms = Geo::SfAtoms;
  static constexpr int SFABytes = SfAtoms * 512;           // 2 KB NVFP4 (own 128 rows)
  static constexpr int SFBBytes = 2 * SfAtoms * 512;       // 4 KB NVFP4 (all 256 rows)
  static constexpr int StageBytes = ABytes + BBytes + SFABytes + SFBBytes;
  static constexpr int StageTx = ATx + BTx + SFABytes + SFBBytes;

  // NVFP4's scale factors take 12 tcgen05.cp per k-tile (twice MXFP4's: 16-element blocks)
  // next to 4 MMAs and their commits.  All of them are issued by the leader CTA, and one warp
  // issues a dependent tcgen05 instruction only every ~40-48 clocks, so a single warp cannot
  // issue a k-tile's 19 instructions within the ~513 clocks its MMAs take.  The work is split
  // between two warps: a copy warp copies SFB and the last SFA atom into SfBufs TMEM buffers,
  // up to SfBufs k-tiles ahead of the MMAs, and the MMA warp copies the other MmaSfaAtoms SFA
  // atoms itself, in order, right before the k-tile's MMAs (11 and 9 instructions per k-tile).
  // The stage's scale factors are loaded first and land on a barrier of their own, so the copy
  // warp need not wait for the stage's A and B.  Measured on B200 at 8192^3, back to back:
  // all 12 copies in the copy warp 231 us, this split 216 us; all 12 in the MMA warp was ~5%
  // slower than the copy warp, and two copy warps slower still.  For MXFP4 the handoff costs
  // more than it saves, so its MMA warp copies everything.
  //
  // OverlapAcc: two accumulator stages that share AccOverlap columns of TMEM (stage s at
  // column s * AccStageStride), one tile per stage in turn, and one scale-factor buffer after
  // them, copied by the MMA warp right before each k-tile's MMAs.  The epilogue reads the
  // shared columns first and releases the accumulator as soon as they are in registers, so the
  // next tile's MMAs start while the epilogue still drains the rest of the previous one.
  static constexpr bool OverlapAcc = OverlapAcc_;
  static constexpr uint32_t AccOverlap = 64;
  static constexpr uint32_t AccStageStride = 256 - AccOverlap;
  static constexpr bool SfCopyWarp = Fmt::SfVec == 16 && !OverlapAcc;
  static constexpr int SfBufs = SfCopyWarp ? 4 : 1;
  static constexpr int NumWarps = SfCopyWarp ? 11 : 10;
  static constexpr int NumThreads = NumWarps * 32;
  static constexpr int ProducerWarp = 0;
  static constexpr int MmaWarp = 1;
  static constexpr int FirstEpiWarp = 2;
  static constexpr int NumEpiWarps = 8;
  static constexpr int SfWarp = 10;              // (SfCopyWarp only)
  static constexpr int MmaSfaAtoms = SfCopyWarp ? SfAtoms - 1 : 0;   // SFA atoms the MMA warp copies

  // TMEM columns: accumulator [0,256); scale factors after it: SFA (4 columns per k-step)
  // then SFB (8 per k-step).
  static constexpr uint32_t TmemCols = 512;
  static constexpr uint32_t AccCol = 0;
  static constexpr uint32_t SfCol = OverlapAcc ? AccStageStride + 256 : 256;
  static constexpr uint32_t SfStride = 12 * SfAtoms;

  // epilogue staging: one 32-row x 64-column BF16 box (4 KB, 128B-swizzled) per epilogue warp
  static constexpr int StoreBoxBytes = 32 * 64 * 2;
  static constexpr int StagingBytes = NumEpiWarps * StoreBoxBytes;

  // stage full/empty, accumulator full/empty, drain, TMEM slot + abort flag, then (copy warp)
  // scale-factor buffer full/empty, the copy warp's drain barrier and the stages' scale-factor
  // full barriers
  static constexpr int BarrierBytes =
      8 * (2 * Stages + 4) + 16 + 8 * (2 * SfBufs + 1) + (SfCopyWarp ? 8 * Stages : 0);
  static constexpr int SmemBytes = Stages * StageBytes + StagingBytes + BarrierBytes + 1024;

  static_assert(SmemBytes <= arch_traits<Arch::kSm100>::max_smem_per_cta, "smem budget");
  static_assert(SfCol + SfBufs * SfStride <= TmemCols, "TMEM budget");
};
using Nvfp4Gemm2SmTraits = Nvfp4Gemm2SmTraitsT<5>;

#if defined(__CUDACC__)

struct Nvfp4Gemm2SmParams {
  CUtensorMap tmap_a;     // A  [M][K/2] bytes, box 128 x 128 B, 128B swizzle
  CUtensorMap tmap_b;     // B  [N][K/2] bytes, box 128 x 128 B, 128B swizzle
  CUtensorMap tmap_sfa;   // SFA [M/128][K/256][2048 B], box one block x one k-tile
  CUtensorMap tmap_sfb;   // SFB [ceil(N/128)][K/256][2048 B], box two blocks x one k-tile
  CUtensorMap tmap_d;     // D  [M][N] bf16, box 32 rows x 64 columns, 128B swizzle
  uint32_t* status;
  float alpha;
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  int raster_m;           // tiles walk raster_m 256-row blocks at a time, all N for each group
  int k_tiles;
  int sf_k_atoms;
  int sf_tail;            // K % 256 != 0: tmap_sfa / tmap_sfb are atom-granular (y = atom)
  // Gather mode: every output tile is also written, with plain 16-byte stores, to up to
  // kMaxGatherPeers further row-major buffers (another GPU's memory mapped into this process,
  // or local memory); peer_d[i] points at this call's first column in buffer i, rows ldd
  // elements apart.  num_peers = 0 is the ordinary GEMM.
  int num_peers;
  int64_t ldd;
  uint8_t* peer_d[kMaxGatherPeers];
};

namespace detail {

// Tile-rows per raster group: a group's rows of A (and SFA) stay in L2 while every column of B
// streams past, so the larger the group the fewer times B is re-read from HBM -- as long as
// the group's A fits the share of the 126 MB L2 given to it here (36 MiB), past which A itself
// is evicted.  Measured on B200: 8192^3 (1.06 MB per tile-row) 245 / 241 / 240 us at groups
// of 8 / 16 / 32; 16384 x 8192 x 28672 (3.8 MB per tile-row) 1.64-1.65 / 1.71 / 1.89 ms.
inline int raster_group_2sm(int K, int tiles_m) {
  const int64_t row_bytes = int64_t(256) * (K / 2 + K / 16);
  int64_t g = (int64_t(36) << 20) / (row_bytes > 0 ? row_bytes : 1);
  if (g > 32) g = 32;
  if (g < 4) g = 4;
  if (g > tiles_m) g = tiles_m;
  if (g < 1) g = 1;
  // the fewest groups of at most g rows, then equal groups: a last group of a single row would
  // stream all of B again for one row (16384 x 8192 x 28672: 1.67 ms at 9 rows, 7 groups + 1)
  const int64_t groups = (tiles_m + g - 1) / g;
  return static_cast<int>((tiles_m + groups - 1) / groups);
}

__device__ __forceinline__ void tile_coords_2sm(int tile, const Nvfp4Gemm2SmParams& p, int& m_blk,
                                                int& n_blk) {
  const int G = p.raster_m;  // raster group, in 256-row tiles
  const int group_tiles = G * p.tiles_n;
  const int group = tile / group_tiles;
  const int first_m = group * G;
  const int rows = min(G, p.tiles_m - first_m);
  const int local = tile - group * group_tiles;
  m_blk = first_m + local % rows;
  n_blk = local / rows;
}

}  // namespace detail

template <class KT, bool kGather = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(KT::NumThreads, 1)
    nvfp4_gemm_2sm_kernel(const __grid_constant__ Nvfp4Gemm2SmParams p) {
#if defined(BLACKHOLE_ARCH_SM100)
  using namespace ptx;
  constexpr int S = KT::Stages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw);

  const uint32_t sA = base;
  const uint32_t sB = sA + S * KT::ABytes;
  const uint32_t sSFA = sB + S * KT::BBytes;
  const uint32_t sSFB = sSFA + S * KT::SFABytes;
  const uint32_t sStage = sSFB + S * KT::SFBBytes;   // epilogue staging boxes
  const uint32_t bars = sStage + KT::StagingBytes;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
  const uint32_t acc_full = bars + 16u * S;
  const uint32_t acc_empty = acc_full + 8u;
  const uint32_t drain_bar = acc_full + 16u;
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + (bars - base) + 16 * S + 32);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sf_full0 = bars + 16u * S + 48u;                 // + 8 b, b < SfBufs
  const uint32_t sf_empty0 = sf_full0 + 8u * KT::SfBufs;          // + 8 b
  const uint32_t sf_drain = sf_full0 + 16u * KT::SfBufs;
  // (copy warp) the stage's scale factors have landed; without a copy warp full_bar covers them
  auto sf_bar = [&](int s) { return KT::SfCopyWarp ? sf_drain + 8u + 8u * s : full_bar(s); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();  // the next kernel may claim SMs as ours exit
  const uint32_t rank = cluster_ctarank();          // 0 = leader, 1 = peer
  const int cluster = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * KT::NumEpiWarps);
    mbar_init(drain_bar, 1);
    if constexpr (KT::SfCopyWarp) {
      for (int b = 0; b < KT::SfBufs; ++b) {
        mbar_init(sf_full0 + 8u * b, 1);
        mbar_init(sf_empty0 + 8u * b, 1);
      }
      mbar_init(sf_drain, 1);
      for (int s = 0; s < S; ++s) mbar_init(sf_bar(s), 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == KT::MmaWarp) {
    tmem_alloc_pair(smem_u32(tmem_slot), KT::TmemCols);
    tmem_relinquish_pair();
  }
  if (warp == KT::ProducerWarp && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    prefetch_tmap(&p.tmap_b);
    prefetch_tmap(&p.tmap_sfa);
    prefetch_tmap(&p.tmap_sfb);
    prefetch_tmap(&p.tmap_d);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the previous kernel in the stream must be complete before global memory is touched
  pdl_wait_prior_grid();

  if (warp == KT::ProducerWarp) {
    // ------------------------------ TMA producer (both CTAs) ------------------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < p.num_tiles; tile += num_clusters) {
        int m_blk, n_blk;
        detail::tile_coords_2sm(tile, p, m_blk, n_blk);
        const int a_row = m_blk * KT::TileM + int(rank) * KT::CtaM;
        const int b_row = n_blk * KT::TileN + int(rank) * KT::CtaN;
        const int sfa_blk = m_blk * 2 + int(rank);
        const int sfb_blk = n_blk * 2;
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (!wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.status, kStatusLoadTimeout)) {
            ok = false;
            break;
          }
          const uint32_t lb = mapa_shared(full_bar(stage), 0);
          const uint32_t ls = mapa_shared(sf_bar(stage), 0);
          if (rank == 0) {
            if constexpr (KT::SfCopyWarp) {
              mbar_arrive_expect_tx(sf_bar(stage), 2u * (KT::SFABytes + KT::SFBBytes));
              mbar_arrive_expect_tx(full_bar(stage), 2u * (KT::ATx + KT::BTx));
            } else {
              mbar_arrive_expect_tx(full_bar(stage), 2u * KT::StageTx);
            }
          }
          // scale factors first (the copy warp waits for them alone), one request per
          // operand: SFA as one 2 KB row, SFB as the pair's two 2 KB rows
          const int sf_y = p.sf_tail ? KT::SfAtoms * kt : kt;
          tma_load_3d_pair(sSFA + stage * KT::SFABytes, &p.tmap_sfa, ls, 0, sf_y, sfa_blk, pol);
          tma_load_3d_pair(sSFB + stage * KT::SFBBytes, &p.tmap_sfb, ls, 0, sf_y, sfb_blk, pol);
          tma_load_2d_pair(sA + stage * KT::ABytes, &p.tmap_a, lb, kt * KT::RowBytes, a_row, pol);
          tma_load_2d_pair(sB + stage * KT::BBytes, &p.tmap_b, lb, kt * KT::RowBytes, b_row, pol);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        for (int s = 0; s < S; ++s) {
          if (issued > s) {
            const int64_t cnt = (issued - 1 - s) / S + 1;
            detail::drain_wait(full_bar(s), uint32_t((cnt - 1) & 1));
            if (KT::SfCopyWarp) detail::drain_wait(sf_bar(s), uint32_t((cnt - 1) & 1));
          }
        }
      }
    }
  } else if (warp == KT::MmaWarp) {
    // ------------------------------ MMA issuer (leader CTA) -------------------------
    // Per k-tile: probe the next stage's barrier, copy this stage's scale factors to TMEM,
    // four MMAs, commit, then consume the probe (falling back to a bounded wait).
    if (rank == 0) {
      constexpr uint32_t idesc = idesc_block_scaled(KT::TileM, KT::TileN, KT::Fmt::AFormat,
                                                    KT::Fmt::BFormat, KT::Fmt::ScaleType);
      const uint32_t acc_full_0 = mapa_shared(acc_full, 0);
      const uint32_t acc_full_1 = mapa_shared(acc_full, 1);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      uint32_t sfbuf = 0;
      int64_t nkt = 0;   // k-tiles issued by this CTA: scale-factor buffer nkt % SfBufs
      bool ok = true;
      bool issued_any = false;
      auto copy_sf = [&](int st, uint32_t b) {
        const uint32_t sfa_s = sSFA + st * KT::SFABytes;
        const uint32_t sfb_s = sSFB + st * KT::SFBBytes;
        const uint32_t ta = tmem + KT::SfCol + KT::SfStride * b;
#pragma unroll
        for (int j = 0; j < KT::SfAtoms; ++j) {
          tc_cp_32x128b_warpx4_pair_w(ta + 4 * j, desc_sf_atom(sfa_s + 512 * j));
          tc_cp_32x128b_warpx4_pair_w(ta + 4 * KT::SfAtoms + 8 * j, desc_sf_atom(sfb_s + 512 * j));
          tc_cp_32x128b_warpx4_pair_w(ta + 4 * KT::SfAtoms + 8 * j + 4,
                                      desc_sf_atom(sfb_s + KT::SFBBytes / 2 + 512 * j));
        }
      };
      for (int tile = cluster; ok && tile < p.num_tiles; tile += num_clusters) {
        // the tile's accumulator: one of the two overlapping stages in turn (OverlapAcc)
        const uint32_t acc_col = KT::OverlapAcc ? (acc_phase ? KT::AccStageStride : 0u) : KT::AccCol;
        if constexpr (KT::OverlapAcc) {
          // first stage, then its scale factors, then the accumulator: the copies run while
          // the epilogue is still releasing the previous tile's shared columns
          if (!wait_bounded_warp(full_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          copy_sf(stage, 0u);
          issued_any = true;
          if (!wait_bounded_warp(acc_empty, acc_phase ^ 1u, abort_flag, p.status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
        } else {
          if (!wait_bounded_warp(acc_empty, acc_phase ^ 1u, abort_flag, p.status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // the first stage of a tile is waited for; each later one is probed one k-tile ahead
          // (A / B and, with the copy warp, the stage's own scale-factor barrier: this warp
          // copies part of SFA from it)
          if (!wait_bounded_warp(full_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout) ||
              (KT::SfCopyWarp &&
               !wait_bounded_warp(sf_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          const int nstage = stage + 1 == S ? 0 : stage + 1;
          const uint32_t nphase = stage + 1 == S ? (phase ^ 1u) : phase;
          const bool more = kt + 1 < p.k_tiles;
          // (a probe issued here is consumed after the MMAs, so its latency stays off the issue
          // chain; a second blocking wait per k-tile measured ~4% slower at 8192^3)
          const uint32_t ready =
              more ? mbar_probe(full_bar(nstage), nphase) &
                         (KT::SfCopyWarp ? mbar_probe(sf_bar(nstage), nphase) : 1u)
                   : 1u;
          if constexpr (KT::SfCopyWarp) {
            sfbuf = uint32_t(nkt % KT::SfBufs);
            // the copy warp's share of buffer sfbuf is in TMEM; this warp copies the first
            // MmaSfaAtoms SFA atoms itself, in order before the MMAs (the stage's scale-factor
            // barrier was acquired with its A / B one k-tile ahead)
            if (!wait_bounded_warp(sf_full0 + 8u * sfbuf, uint32_t((nkt / KT::SfBufs) & 1),
                                   abort_flag, p.status, kStatusMmaTimeout)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sfa_s = sSFA + stage * KT::SFABytes;
            const uint32_t ta0 = tmem + KT::SfCol + KT::SfStride * sfbuf;
#pragma unroll
            for (int j = 0; j < KT::MmaSfaAtoms; ++j)
              tc_cp_32x128b_warpx4_pair_w(ta0 + 4 * j, desc_sf_atom(sfa_s + 512 * j));
          } else if (!KT::OverlapAcc || kt > 0) {
            copy_sf(stage, sfbuf);
          }
          const uint64_t adesc = desc_kmajor<KT::RowBytes>(sA + stage * KT::ABytes);
          const uint64_t bdesc = desc_kmajor<KT::RowBytes>(sB + stage * KT::BBytes);
          const uint32_t ta = tmem + KT::SfCol + KT::SfStride * sfbuf;
#pragma unroll
          for (int j = 0; j < KT::KSteps; ++j) {
            const int at = j / KT::StepsPerAtom;
            const uint32_t sid = KT::Geo::sf_id(j);   // byte in the entry
            tc_mma_bs_pair_w<typename KT::Fmt>(
                tmem + acc_col, adesc + 2 * j, bdesc + 2 * j, idesc_with_sf_id(idesc, sid),
                sf_tmem_addr(ta + 4 * at, sid), sf_tmem_addr(ta + 4 * KT::SfAtoms + 8 * at, sid),
                (kt | j) != 0 ? 1u : 0u);
          }
          tc_commit_pair_w(mapa_shared(empty_bar(stage), 0));
          tc_commit_pair_w(mapa_shared(empty_bar(stage), 1));
          if constexpr (KT::SfCopyWarp) tc_commit_pair_w(mapa_shared(sf_empty0 + 8u * sfbuf, 0));
          ++nkt;
          issued_any = true;
          stage = nstage;
          phase = nphase;
          if (more) {
            if (!__all_sync(0xFFFFFFFFu, ready != 0u) &&
                (!wait_bounded_warp(full_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout) ||
                 (KT::SfCopyWarp &&
                  !wait_bounded_warp(sf_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout)))) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
        }
        if (!ok) break;
        tc_commit_pair_w(acc_full_0);
        tc_commit_pair_w(acc_full_1);
        acc_phase ^= 1u;
      }
      if (!ok && issued_any) {
        tc_commit_pair_w(mapa_shared(drain_bar, 0));
        detail::drain_wait(drain_bar, 0);
      }
      __syncwarp();
    }
  } else if (KT::SfCopyWarp && warp == KT::SfWarp) {
    // ------------------------------ scale-factor copier (leader CTA) ----------------
    // k-tile n: wait until the MMAs of k-tile n - SfBufs have released TMEM buffer n % SfBufs
    // and stage n's scale factors have landed, copy its SFB and its last SFA atoms (the MMA
    // warp copies the first MmaSfaAtoms) into that buffer, commit.
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t nkt = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < p.num_tiles; tile += num_clusters) {
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          const uint32_t b = uint32_t(nkt % KT::SfBufs);
          if (!wait_bounded_warp(sf_empty0 + 8u * b, uint32_t(((nkt / KT::SfBufs) & 1) ^ 1),
                                 abort_flag, p.status, kStatusMmaTimeout) ||
              !wait_bounded_warp(sf_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_s = sSFA + stage * KT::SFABytes;
          const uint32_t sfb_s = sSFB + stage * KT::SFBBytes;
          const uint32_t ta = tmem + KT::SfCol + KT::SfStride * b;
#pragma unroll
          for (int j = 0; j < KT::SfAtoms; ++j) {
            if (j >= KT::MmaSfaAtoms)
              tc_cp_32x128b_warpx4_pair_w(ta + 4 * j, desc_sf_atom(sfa_s + 512 * j));
            tc_cp_32x128b_warpx4_pair_w(ta + 4 * KT::SfAtoms + 8 * j, desc_sf_atom(sfb_s + 512 * j));
            tc_cp_32x128b_warpx4_pair_w(ta + 4 * KT::SfAtoms + 8 * j + 4,
                                        desc_sf_atom(sfb_s + KT::SFBBytes / 2 + 512 * j));
          }
          tc_commit_pair_w(mapa_shared(sf_full0 + 8u * b, 0));
          ++nkt;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (nkt > 0) {   // every copy issued here has landed before TMEM is released
        tc_commit_pair_w(mapa_shared(sf_drain, 0));
        detail::drain_wait(sf_drain, 0);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------ epilogue (both CTAs) ----------------------------
    const int q = warp & 3;
    const int half = (warp - KT::FirstEpiWarp) >> 2;
    const uint32_t leader_acc_empty = mapa_shared(acc_empty, 0);
    uint32_t acc_phase = 0;
    for (int tile = cluster; tile < p.num_tiles; tile += num_clusters) {
      int m_blk, n_blk;
      detail::tile_coords_2sm(tile, p, m_blk, n_blk);
      if (!wait_bounded_warp(acc_full, acc_phase, abort_flag, p.status, kStatusEpilogueTimeout)) break;
      tc_fence_after();
      uint32_t v0[32], v1[32], v2[32], v3[32];
      // Measured on B200: the two-SM kind::mxf8f6f4 MMA (N = 256) leaves output column n in
      // accumulator column n XOR 32 (32-column groups swapped pairwise inside each half; lanes
      // and halves as for kind::mxf4nvf4), so that kind reads the groups crosswise.
      constexpr uint32_t x = KT::Fmt::Kind == MmaKind::kMxf8f6f4 ? 32u : 0u;
      const uint32_t acc_col = KT::OverlapAcc ? (acc_phase ? KT::AccStageStride : 0u) : KT::AccCol;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * q) << 16) + acc_col + 128 * half;
      if constexpr (KT::OverlapAcc) {
        // Stage 0 shares its last 64 columns with stage 1, stage 1 its first 64 with stage 0.
        // The warps of the half that holds them read those first and release the accumulator;
        // the other half's warps release it at once (the next tile's MMAs never touch their
        // columns, and the tile after that waits for their release of the next tile).
        const bool shared_hi = acc_phase == 0u;
        const bool holds = (half == 1) == shared_hi;
        if (!holds) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_acc_empty);
        }
        if (shared_hi) {
          tmem_ld_32x32b_x32(t_row + (64 ^ x), v2);
          tmem_ld_32x32b_x32(t_row + (96 ^ x), v3);
        } else {
          tmem_ld_32x32b_x32(t_row + (0 ^ x), v0);
          tmem_ld_32x32b_x32(t_row + (32 ^ x), v1);
        }
        tmem_ld_wait();
        if (holds) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_acc_empty);
        }
        if (shared_hi) {
          tmem_ld_32x32b_x32(t_row + (0 ^ x), v0);
          tmem_ld_32x32b_x32(t_row + (32 ^ x), v1);
        } else {
          tmem_ld_32x32b_x32(t_row + (64 ^ x), v2);
          tmem_ld_32x32b_x32(t_row + (96 ^ x), v3);
        }
        tmem_ld_wait();
        reg_fence(v0);
        reg_fence(v1);
        reg_fence(v2);
        reg_fence(v3);
      } else {
        tmem_ld_32x32b_x32(t_row + (0 ^ x), v0);
        tmem_ld_32x32b_x32(t_row + (32 ^ x), v1);
        tmem_ld_32x32b_x32(t_row + (64 ^ x), v2);
        tmem_ld_32x32b_x32(t_row + (96 ^ x), v3);
        tmem_ld_wait();
        reg_fence(v0);
        reg_fence(v1);
        reg_fence(v2);
        reg_fence(v3);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(leader_acc_empty);
      }
      acc_phase ^= 1u;

      // alpha * acc -> BF16 -> this warp's swizzled staging box -> TMA store, 64 columns at
      // a time.  Lane i owns row i of the box; its 16-byte chunk c lands at chunk c ^ (i % 8)
      // of the 128-byte row, the layout CU_TENSOR_MAP_SWIZZLE_128B expects.
      const int row0 = m_blk * KT::TileM + int(rank) * KT::CtaM + 32 * q;
      const int col0 = n_blk * KT::TileN + 128 * half;
      const uint32_t box = sStage + (warp - KT::FirstEpiWarp) * KT::StoreBoxBytes;
      const uint32_t my_row = box + lane * 128;
      const float a = p.alpha;
      const uint64_t pol_d = l2_policy_evict_first();   // keep A / B resident in L2
      auto stage_store = [&](uint32_t (&va)[32], uint32_t (&vb)[32], int u) {
        if (lane == 0) bulk_wait_group_read<0>();   // previous box has been read out
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t (&v)[32] = c < 4 ? va : vb;
          const int i = (c & 3) * 8;
          st_shared_v4(my_row + ((c ^ (lane & 7)) << 4),
                       detail::pack_bf16x2(a * __uint_as_float(v[i + 0]), a * __uint_as_float(v[i + 1])),
                       detail::pack_bf16x2(a * __uint_as_float(v[i + 2]), a * __uint_as_float(v[i + 3])),
                       detail::pack_bf16x2(a * __uint_as_float(v[i + 4]), a * __uint_as_float(v[i + 5])),
                       detail::pack_bf16x2(a * __uint_as_float(v[i + 6]), a * __uint_as_float(v[i + 7])));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < p.M && col0 + 64 * u < p.N) {
          tma_store_2d(&p.tmap_d, box, col0 + 64 * u, row0, pol_d);
          bulk_commit_group();
        }
        if constexpr (kGather) {
          // the same box to every further buffer: 8 lanes per 128-byte row segment
#pragma unroll 1
          for (int it = 0; it < 8; ++it) {
            const int r = it * 4 + (lane >> 3);
            const int ch = lane & 7;
            const int grow = row0 + r;
            const int gcol = col0 + 64 * u + 8 * ch;
            if (grow < p.M && gcol < p.N) {
              const uint4 v = ld_shared_v4(box + r * 128 + ((ch ^ (r & 7)) << 4));
              const int64_t off = (int64_t(grow) * p.ldd + gcol) * 2;
              for (int q = 0; q < p.num_peers; ++q)
                *reinterpret_cast<uint4*>(p.peer_d[q] + off) = v;
            }
          }
        }
      };
      stage_store(v0, v1, 0);
      stage_store(v2, v3, 1);
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its partner may still signal it
  if (warp == KT::MmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, KT::TmemCols);
  }
#endif  // BLACKHOLE_ARCH_SM100
}

namespace detail {

template <class KT>
inline cudaError_t launch_2sm(int M, int N, int K, const void* A, const void* SFA, const void* B,
                              const void* SFB, void* D, float alpha, DeviceState* st, int dev,
                              cudaStream_t stream, const GatherSpec* g = nullptr) {
  // gather mode has its own instantiation (NVFP4 only: the gather entry point's format), so
  // the plain GEMM carries none of its code
  constexpr bool kCanGather = std::is_same_v<typename KT::Fmt, Nvfp4Format>;
  if (g && !kCanGather) return cudaErrorInvalidValue;
  auto* kernel = nvfp4_gemm_2sm_kernel<KT, false>;
  if constexpr (kCanGather)
    if (g) kernel = nvfp4_gemm_2sm_kernel<KT, true>;
  cudaError_t e = set_smem_once(kernel, KT::SmemBytes, dev);
  if (e != cudaSuccess) return e;
  Nvfp4Gemm2SmParams p;
  e = make_a_tmap<typename KT::Fmt>(&p.tmap_a, A, M, K, KT::CtaM);
  if (e != cudaSuccess) return e;
  e = make_b_tmap<typename KT::Fmt>(&p.tmap_b, B, N, K, KT::CtaN);
  if (e != cudaSuccess) return e;
  // K % 256 != 0: 4 rows of 512 B per block, so that the K tail reads zeros (slower per k-tile)
  p.sf_tail = K % KT::TileK != 0;
  e = p.sf_tail ? make_sf_tmap_atoms(&p.tmap_sfa, SFA, M, K, 1, KT::SfAtoms, KT::SFVecSize)
                : make_sf_tmap_ktile(&p.tmap_sfa, SFA, M, K, 1, 1, KT::SfAtoms, KT::SFVecSize);
  if (e != cudaSuccess) return e;
  e = p.sf_tail ? make_sf_tmap_atoms(&p.tmap_sfb, SFB, N, K, 2, KT::SfAtoms, KT::SFVecSize)
                : make_sf_tmap_ktile(&p.tmap_sfb, SFB, N, K, 2, 1, KT::SfAtoms, KT::SFVecSize);
  if (e != cudaSuccess) return e;
  p.num_peers = 0;
  p.ldd = N;
  if (g) {
    uint8_t* own = static_cast<uint8_t*>(g->dst[0]) + g->col0 * 2;
    e = make_d_tmap(&p.tmap_d, own, M, N, 64, g->ldd);
    p.num_peers = g->ndst - 1;
    p.ldd = g->ldd;
    for (int i = 0; i < kMaxGatherPeers; ++i)
      p.peer_d[i] = i + 1 < g->ndst ? static_cast<uint8_t*>(g->dst[i + 1]) + g->col0 * 2 : nullptr;
  } else {
    e = make_d_tmap(&p.tmap_d, D, M, N);
  }
  if (e != cudaSuccess) return e;
  p.status = st->status;
  p.alpha = alpha;
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_m = (M + KT::TileM - 1) / KT::TileM;
  p.tiles_n = (N + KT::TileN - 1) / KT::TileN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.raster_m = detail::raster_group_2sm(K, p.tiles_m);
  p.k_tiles = (K + KT::TileK - 1) / KT::TileK;
  p.sf_k_atoms = static_cast<int>(sf_k_atoms_vs(K, KT::SFVecSize));
  // Persistent grid = the number of 2-CTA clusters that can be resident at once.  GPCs with
  // an odd number of usable SMs leave an SM idle, so this is below num_sms / 2; launching
  // num_sms / 2 clusters would run the excess as a second wave.
  static std::mutex mu;
  static int resident[64] = {0};
  int clusters = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (resident[dev & 63] == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(st->num_sms & ~1), 1, 1);
      cfg.blockDim = dim3(KT::NumThreads, 1, 1);
      cfg.dynamicSmemBytes = KT::SmemBytes;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
      if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = st->num_sms / 2;
      }
      resident[dev & 63] = n;
    }
    clusters = resident[dev & 63];
  }
  if (p.num_tiles < clusters) clusters = p.num_tiles;
  e = launch_pdl(kernel, dim3(2 * clusters), dim3(KT::NumThreads), KT::SmemBytes,
                 stream, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace detail

#endif  // __CUDACC__

}  // namespace blackhole::sm100
