#pragma once

// =====================================================================================
// blackhole / sm100 / NVFP4 GEMM, one-SM schedule (cta_group::1, 128 x 256 tiles)
// -------------------------------------------------------------------------------------
// Persistent CTA per SM, 10 warps:
//   warp 0 (TMA)   : for each k-tile of 256 K: TMA 128x128B of A and 256x128B of B
//                    (128B swizzle) and bulk-copy the 2 KB + 4 KB scale-factor atoms into a
//                    4-stage shared-memory ring; full/empty mbarrier pair per stage.
//   warp 1 (MMA)   : tcgen05.cp the scale factors smem -> TMEM, then four
//                    tcgen05.mma.kind::mxf4nvf4.block_scale (128x256x64 each) per k-tile
//                    into a 128 x 256 FP32 accumulator in TMEM; tcgen05.commit frees the
//                    smem stage; after the last k-tile it signals the epilogue.
//   warps 2-9 (epi): tcgen05.ld the accumulator (two warps per 32-lane sub-partition, 128
//                    columns each), release TMEM to the MMA warp at once, then alpha * acc
//                    -> BF16 through a 1 KB swizzled shared-memory box per warp and TMA
//                    tensor stores while the next tile's mainloop runs.
// Used for small problems; large ones take the two-SM schedule (nvfp4_gemm_2sm.hpp).
// =====================================================================================

#include <blackhole/sm100/block_scale_format.hpp>
#include <blackhole/sm100/nvfp4_gemm_common.hpp>

namespace blackhole::sm100 {

// =====================================================================================
// 1. Compile-time configuration
// =====================================================================================
template <int Stages_ = 4, class Fmt_ = Nvfp4Format>
struct Nvfp4GemmTraitsT {
  using Fmt = Fmt_;
  using Geo = BlockScaleGeometry<Fmt>;
  static constexpr int SFVecSize = Fmt::SfVec;   // elements per scale factor (16 or 32)

  static constexpr int TileM = 128;              // UMMA M (one CTA, TMEM lanes)
  static constexpr int TileN = 256;              // UMMA N
  static constexpr int TileK = Fmt::TileK;       // elements per k-tile (128-byte smem rows)
  static constexpr int KSteps = Geo::KSteps;     // 4 MMAs per k-tile
  static constexpr int Stages = Stages_;

  static constexpr int RowBytes = Geo::RowBytes;                    // 128
  static constexpr int ABytes = TileM * RowBytes;                   // 16 KB
  static constexpr int BBytes = TileN * RowBytes;                   // 32 KB
  // bytes the A / B loads of a k-tile complete on the stage barrier (global bytes: an
  // expanded 4-bit B fills twice its size in shared memory)
  static constexpr int ATx = TileM * Geo::ARowTx;
  static constexpr int BTx = TileN * Geo::BRowTx;
  // 512-byte scale-factor atoms per 128 rows and k-tile: 4 (NVFP4), 2 (MXFP4), 1 (MXFP8 x
  // MXFP4); k-step j reads atom j / StepsPerAtom from scale-factor ID Geo::sf_id(j).
  static constexpr int StepsPerAtom = Geo::StepsPerAtom;
  static constexpr int SfAtoms = Geo::SfAtoms;
  static constexpr int SFABytes = (TileM / 128) * SfAtoms * 512;    // 2 KB (NVFP4)
  static constexpr int SFBBytes = (TileN / 128) * SfAtoms * 512;    // 4 KB (NVFP4)
  static constexpr int StageBytes = ABytes + BBytes + SFABytes + SFBBytes;

  static constexpr int NumWarps = 10;
  static constexpr int NumThreads = NumWarps * 32;
  static constexpr int ProducerWarp = 0;
  static constexpr int MmaWarp = 1;
  static constexpr int FirstEpiWarp = 2;
  static constexpr int NumEpiWarps = 8;

  // TMEM columns: accumulator [0,256); scale factors after it: SFA (4 columns per k-step)
  // then SFB (8 per k-step).
  static constexpr uint32_t TmemCols = 512;
  static constexpr uint32_t AccCol = 0;
  static constexpr uint32_t SfCol = 256;
  static constexpr uint32_t SfStride = 12 * SfAtoms;

  // epilogue staging: one 32-row x 16-column BF16 box (1 KB, 32B-swizzled) per epilogue warp
  static constexpr int StoreBoxBytes = 32 * 16 * 2;
  static constexpr int StagingBytes = NumEpiWarps * StoreBoxBytes;

  // shared memory: stage ring + staging + barriers (+1 KB to align the ring to 1024 B)
  static constexpr int BarrierBytes = 8 * (2 * Stages + 4) + 16;
  static constexpr int SmemBytes = Stages * StageBytes + StagingBytes + BarrierBytes + 1024;

  static constexpr int RasterGroupM = 16;  // tiles walk 16 M-blocks at a time (L2 reuse)

  static_assert(SmemBytes <= arch_traits<Arch::kSm100>::max_smem_per_cta, "smem budget");
  static_assert(SfCol + 2 * SfStride <= TmemCols, "TMEM budget");
};
using Nvfp4GemmTraits = Nvfp4GemmTraitsT<4>;

#if defined(__CUDACC__)

// =====================================================================================
// 2. Kernel
// =====================================================================================
struct Nvfp4GemmParams {
  CUtensorMap tmap_a;   // A as uint8 [M][K/2], box 128 x 128 B, 128B swizzle
  CUtensorMap tmap_b;   // B as uint8 [N][K/2], box 256 x 128 B, 128B swizzle
  CUtensorMap tmap_d;   // D bf16 [M][N], box 32 rows x 16 columns, 32B swizzle
  const uint8_t* sfa;
  const uint8_t* sfb;
  uint32_t* status;
  float alpha;
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  int k_tiles;
  int sf_k_atoms;       // 512-byte SF atoms along K per 128-row block
  int n_blocks128;      // 128-row blocks of B (and of SFB): ceil(N / 128)
  int sf_tail;          // K % TileK != 0: scale factors through the atom-granular tensor maps
  CUtensorMap tmap_sfa; // (sf_tail only) SFA [M/128][atoms][512 B], box 4 atoms x 1 block
  CUtensorMap tmap_sfb; // (sf_tail only) SFB [N/128][atoms][512 B], box 4 atoms x 2 blocks
};


namespace detail {

template <class KT>
__device__ __forceinline__ void tile_coords(int tile, const Nvfp4GemmParams& p, int& m_blk,
                                            int& n_blk) {
  const int group_tiles = KT::RasterGroupM * p.tiles_n;
  const int group = tile / group_tiles;
  const int first_m = group * KT::RasterGroupM;
  const int rows = min(KT::RasterGroupM, p.tiles_m - first_m);
  const int local = tile - group * group_tiles;
  m_blk = first_m + local % rows;
  n_blk = local / rows;
}

}  // namespace detail

template <class KT>
__global__ void __launch_bounds__(KT::NumThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ Nvfp4GemmParams p) {
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
  const uint32_t sStage = sSFB + S * KT::SFBBytes;  // epilogue staging boxes
  const uint32_t bars = sStage + KT::StagingBytes;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
  const uint32_t acc_full = bars + 16u * S;
  const uint32_t acc_empty = acc_full + 8u;
  const uint32_t drain_bar = acc_full + 16u;
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + (bars - base) + 16 * S + 32);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();  // the next kernel may claim SMs as ours exit

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, KT::NumEpiWarps);
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
    prefetch_tmap(&p.tmap_a);
    prefetch_tmap(&p.tmap_b);
    prefetch_tmap(&p.tmap_d);
    if (p.sf_tail) {
      prefetch_tmap(&p.tmap_sfa);
      prefetch_tmap(&p.tmap_sfb);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the previous kernel in the stream must be complete before global memory is touched
  pdl_wait_prior_grid();

  if (warp == KT::ProducerWarp) {
    // ------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();
      // With one M tile (M <= 128: decode widths) every byte of B is read once: streaming it
      // evict-first keeps A and the scale factors in L2 (measured on B200 at N = 28672,
      // K = 8192: M = 32 / 64 / 128 took 2.5-3.5% less time).  A second M tile re-reads B.
      const uint64_t pol_b = p.tiles_m == 1 ? l2_policy_evict_first() : l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        int m_blk, n_blk;
        detail::tile_coords<KT>(tile, p, m_blk, n_blk);
        const bool sfb_hi = (2 * n_blk + 1) < p.n_blocks128;
        const uint32_t bytes =
            KT::ATx + KT::BTx + KT::SFABytes +
            ((sfb_hi || p.sf_tail) ? KT::SFBBytes : KT::SFBBytes / 2);
        const uint8_t* sfa_src = p.sfa + (int64_t(m_blk) * p.sf_k_atoms) * 512;
        const uint8_t* sfb_src0 = p.sfb + (int64_t(2 * n_blk) * p.sf_k_atoms) * 512;
        const uint8_t* sfb_src1 = sfb_src0 + int64_t(p.sf_k_atoms) * 512;
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (!wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.status,
                            kStatusLoadTimeout)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, bytes);
          tma_load_2d(sA + stage * KT::ABytes, &p.tmap_a, fb, kt * KT::RowBytes, m_blk * KT::TileM,
                      pol_a);
          tma_load_2d(sB + stage * KT::BBytes, &p.tmap_b, fb, kt * KT::RowBytes, n_blk * KT::TileN,
                      pol_b);
          const int64_t k_off = int64_t(kt) * KT::SfAtoms * 512;
          if (p.sf_tail) {  // atoms past K (and blocks past N) read zeros
            tma_load_3d(sSFA + stage * KT::SFABytes, &p.tmap_sfa, fb, 0, KT::SfAtoms * kt, m_blk,
                        pol_a);
            tma_load_3d(sSFB + stage * KT::SFBBytes, &p.tmap_sfb, fb, 0, KT::SfAtoms * kt,
                        2 * n_blk, pol_b);
          } else {
            bulk_load(sSFA + stage * KT::SFABytes, sfa_src + k_off, KT::SFABytes, fb, pol_a);
            bulk_load(sSFB + stage * KT::SFBBytes, sfb_src0 + k_off, KT::SFBBytes / 2, fb, pol_b);
            if (sfb_hi)
              bulk_load(sSFB + stage * KT::SFBBytes + KT::SFBBytes / 2, sfb_src1 + k_off,
                        KT::SFBBytes / 2, fb, pol_b);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the copies already in flight land before the CTA goes away.
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
    // Per k-tile: probe the next stage's barrier, copy this stage's scale factors to TMEM,
    // four MMAs, commit, then consume the probe (falling back to a bounded wait).
    constexpr uint32_t idesc = idesc_block_scaled(KT::TileM, KT::TileN, KT::Fmt::AFormat,
                                                  KT::Fmt::BFormat, KT::Fmt::ScaleType);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_phase = 0;
    const uint32_t sfbuf = 0;
    bool ok = true;
    bool issued_any = false;
    auto copy_sf = [&](int st, uint32_t b) {
      const uint32_t sfa_s = sSFA + st * KT::SFABytes;
      const uint32_t sfb_s = sSFB + st * KT::SFBBytes;
      const uint32_t ta = tmem + KT::SfCol + KT::SfStride * b;
#pragma unroll
      for (int j = 0; j < KT::SfAtoms; ++j) {
        tc_cp_32x128b_warpx4_w(ta + 4 * j, desc_sf_atom(sfa_s + 512 * j));
        tc_cp_32x128b_warpx4_w(ta + 4 * KT::SfAtoms + 8 * j, desc_sf_atom(sfb_s + 512 * j));
        tc_cp_32x128b_warpx4_w(ta + 4 * KT::SfAtoms + 8 * j + 4,
                               desc_sf_atom(sfb_s + KT::SFBBytes / 2 + 512 * j));
      }
    };
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      if (!wait_bounded_warp(acc_empty, acc_phase ^ 1u, abort_flag, p.status, kStatusMmaTimeout)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // the first stage of a tile is waited for; each later one is probed one k-tile ahead
      if (!wait_bounded_warp(full_bar(stage), phase, abort_flag, p.status, kStatusMmaTimeout)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        const int nstage = stage + 1 == S ? 0 : stage + 1;
        const uint32_t nphase = stage + 1 == S ? (phase ^ 1u) : phase;
        const bool more = kt + 1 < p.k_tiles;
        const uint32_t ready = more ? mbar_probe(full_bar(nstage), nphase) : 1u;
        copy_sf(stage, sfbuf);
        const uint64_t adesc = desc_kmajor<KT::RowBytes>(sA + stage * KT::ABytes);
        const uint64_t bdesc = desc_kmajor<KT::RowBytes>(sB + stage * KT::BBytes);
        const uint32_t ta = tmem + KT::SfCol + KT::SfStride * sfbuf;
#pragma unroll
        for (int j = 0; j < KT::KSteps; ++j) {
          // +32 bytes of K per step inside the swizzled row (descriptor units: 16 B)
          const int at = j / KT::StepsPerAtom;
          const uint32_t sid = KT::Geo::sf_id(j);   // byte in the entry
          tc_mma_bs_w<typename KT::Fmt>(
              tmem + KT::AccCol, adesc + 2 * j, bdesc + 2 * j, idesc_with_sf_id(idesc, sid),
              sf_tmem_addr(ta + 4 * at, sid), sf_tmem_addr(ta + 4 * KT::SfAtoms + 8 * at, sid),
              (kt | j) != 0 ? 1u : 0u);
        }
        tc_commit_w(empty_bar(stage));
        issued_any = true;
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
      tc_commit_w(acc_full);
      acc_phase ^= 1u;
    }
    if (!ok && issued_any) {
      // wait for the MMAs in flight before TMEM is released
      tc_commit_w(drain_bar);
      detail::drain_wait(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ----------------------------------------
    const int q = warp & 3;                                   // TMEM lane quadrant
    const int half = (warp - KT::FirstEpiWarp) >> 2;          // column half of the tile
    const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * q) << 16) + KT::AccCol + 128 * half;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int m_blk, n_blk;
      detail::tile_coords<KT>(tile, p, m_blk, n_blk);
      if (!wait_bounded_warp(acc_full, acc_phase, abort_flag, p.status, kStatusEpilogueTimeout)) break;
      tc_fence_after();
      uint32_t v0[32], v1[32], v2[32], v3[32];
      tmem_ld_32x32b_x32(t_row + 0, v0);
      tmem_ld_32x32b_x32(t_row + 32, v1);
      tmem_ld_32x32b_x32(t_row + 64, v2);
      tmem_ld_32x32b_x32(t_row + 96, v3);
      tmem_ld_wait();
      reg_fence(v0);
      reg_fence(v1);
      reg_fence(v2);
      reg_fence(v3);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      acc_phase ^= 1u;

      // alpha * acc -> BF16 -> this warp's 1 KB staging box -> TMA store, 16 columns at a
      // time.  Lane i owns row i (32 bytes); its 16-byte chunk c lands at chunk
      // c ^ ((i / 4) % 2), the layout CU_TENSOR_MAP_SWIZZLE_32B expects.
      const int row0 = m_blk * KT::TileM + 32 * q;
      const int col0 = n_blk * KT::TileN + 128 * half;
      const uint32_t box = sStage + (warp - KT::FirstEpiWarp) * KT::StoreBoxBytes;
      const uint32_t my_row = box + lane * 32;
      const uint32_t sw = (lane >> 2) & 1;
      const float a = p.alpha;
      const bool live = row0 < p.M && col0 < p.N;
      const uint64_t pol_d = l2_policy_evict_first();   // keep A / B resident in L2
      auto stage_store = [&](uint32_t (&v)[32], int c32) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (lane == 0) bulk_wait_group_read<0>();   // previous box has been read out
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int i = 16 * h + 8 * c;
            st_shared_v4(my_row + ((c ^ sw) << 4),
                         detail::pack_bf16x2(a * __uint_as_float(v[i + 0]), a * __uint_as_float(v[i + 1])),
                         detail::pack_bf16x2(a * __uint_as_float(v[i + 2]), a * __uint_as_float(v[i + 3])),
                         detail::pack_bf16x2(a * __uint_as_float(v[i + 4]), a * __uint_as_float(v[i + 5])),
                         detail::pack_bf16x2(a * __uint_as_float(v[i + 6]), a * __uint_as_float(v[i + 7])));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && live && col0 + c32 + 16 * h < p.N) {
            tma_store_2d(&p.tmap_d, box, col0 + c32 + 16 * h, row0, pol_d);
            bulk_commit_group();
          }
        }
      };
      stage_store(v0, 0);
      stage_store(v1, 32);
      stage_store(v2, 64);
      stage_store(v3, 96);
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
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
inline cudaError_t launch_1sm(int M, int N, int K, const void* A, const void* SFA, const void* B,
                              const void* SFB, void* D, float alpha, DeviceState* st, int dev,
                              cudaStream_t stream) {
  cudaError_t e = set_smem_once(nvfp4_gemm_kernel<KT>, KT::SmemBytes, dev);
  if (e != cudaSuccess) return e;
  Nvfp4GemmParams p;
  e = make_a_tmap<typename KT::Fmt>(&p.tmap_a, A, M, K, KT::TileM);
  if (e != cudaSuccess) return e;
  e = make_b_tmap<typename KT::Fmt>(&p.tmap_b, B, N, K, KT::TileN);
  if (e != cudaSuccess) return e;
  e = make_d_tmap(&p.tmap_d, D, M, N, 16);
  if (e != cudaSuccess) return e;
  p.sfa = static_cast<const uint8_t*>(SFA);
  p.sfb = static_cast<const uint8_t*>(SFB);
  p.status = st->status;
  p.alpha = alpha;
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_m = (M + KT::TileM - 1) / KT::TileM;
  p.tiles_n = (N + KT::TileN - 1) / KT::TileN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_tiles = (K + KT::TileK - 1) / KT::TileK;
  p.sf_k_atoms = static_cast<int>(sf_k_atoms_vs(K, KT::SFVecSize));
  p.n_blocks128 = (N + 127) / 128;
  p.sf_tail = K % KT::TileK != 0;
  if (p.sf_tail) {
    e = make_sf_tmap_atoms(&p.tmap_sfa, SFA, M, K, 1, KT::SfAtoms, KT::SFVecSize);
    if (e != cudaSuccess) return e;
    e = make_sf_tmap_atoms(&p.tmap_sfb, SFB, N, K, 2, KT::SfAtoms, KT::SFVecSize);
    if (e != cudaSuccess) return e;
  }
  const int grid = p.num_tiles < st->num_sms ? p.num_tiles : st->num_sms;
  e = launch_pdl(nvfp4_gemm_kernel<KT>, dim3(grid), dim3(KT::NumThreads), KT::SmemBytes, stream, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace detail

#endif  // __CUDACC__

}  // namespace blackhole::sm100
