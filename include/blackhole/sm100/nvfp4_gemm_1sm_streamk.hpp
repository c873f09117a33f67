#pragma once

// =====================================================================================
// blackhole / sm100 / NVFP4 GEMM, one-SM schedule split stream-K (every SM streams)
// -------------------------------------------------------------------------------------
// The one-SM schedule (nvfp4_gemm_1sm.hpp) gives each CTA whole 128 x 256 tiles.  When there
// are fewer tiles than SMs -- decode-sized M with N = 28672 has 112 -- a third of the SMs idle
// and the weight stream runs at 112 CTAs' rate.  This variant keeps the tile, the ring, the
// TMEM layout and the epilogue, and splits the (tile, k-tile) units into one contiguous range
// per persistent CTA:
//
//   * units run tile-major (all k-tiles of a tile, then the next tile); CTA c takes units
//     [start(c), start(c+1)); its range is whole tiles plus the tail of one tile and the head
//     of another, walked from its end backwards in tile segments;
//   * a tile split across CTAs is finished by the CTA that owns its last k-tile: the others
//     (which reach it first, walking backwards) park FP32 partials in the workspace and raise a
//     flag per epilogue warp; the finisher's matching warp adds them in a fixed order (so the
//     result is deterministic) and writes BF16;
//   * ranges go to CTAs in the order they start (a ticket taken at entry, before the
//     programmatic-launch trigger), so a finisher only waits for CTAs that already run;
//   * flags carry a per-launch tag (the generation word next to the ticket, advanced once per
//     launch), so a launch that gave up on a bounded wait leaves nothing a later one accepts.
//
// The workspace layout is the skinny schedule's (flags, ticket, generation, then one partial
// slot per CTA), with a 128 KB slot: 128 rows x 256 columns of FP32, stored so that a warp's
// 32 rows x 4 columns are one 512-byte line.
// =====================================================================================

#include <blackhole/sm100/nvfp4_gemm_1sm.hpp>
#include <blackhole/sm100/nvfp4_gemm_skinny.hpp>

namespace blackhole::sm100 {

// Workspace bytes of the stream-K one-SM schedule on a device with num_sms SMs.
constexpr int64_t nvfp4_1sm_streamk_workspace_bytes(int num_sms) {
  return nvfp4_skinny_flag_bytes(num_sms) + int64_t(num_sms) * 128 * 256 * 4;
}

#if defined(__CUDACC__)

struct Nvfp4StreamKParams {
  Nvfp4GemmParams g;    // tensor maps, shapes, tile counts, scale-factor pointers
  float* ws;            // [grid][128 KB] partials
  uint32_t* flags;      // [grid][8]
  uint32_t* ticket;     // [0] entry counter, [1] launch generation
  uint64_t partial_wait_ns;
  int64_t units;        // num_tiles * k_tiles
  int grid;
};

namespace streamk_detail {

__device__ __forceinline__ int64_t range_start(const Nvfp4StreamKParams& p, int t) {
  return int64_t(t) * p.units / p.grid;
}

struct Segment {
  int tile, kt0, kt1;
};

// A CTA's range, walked from its end backwards one tile segment at a time.
struct Walk {
  int64_t begin, u;
  int KT;
  __device__ __forceinline__ bool next(Segment& s) {
    if (u <= begin) return false;
    const int tile = static_cast<int>((u - 1) / KT);
    const int64_t t0 = int64_t(tile) * KT;
    const int64_t sb = begin > t0 ? begin : t0;
    s.tile = tile;
    s.kt0 = static_cast<int>(sb - t0);
    s.kt1 = static_cast<int>(u - t0);
    u = sb;
    return true;
  }
};

__device__ __forceinline__ Walk walk(const Nvfp4StreamKParams& p, int c) {
  Walk w;
  w.begin = range_start(p, c);
  w.u = range_start(p, c + 1);
  w.KT = p.g.k_tiles;
  return w;
}

__device__ __forceinline__ void tile_mn(const Nvfp4GemmParams& g, int tile, int& m_blk, int& n_blk) {
  m_blk = tile % g.tiles_m;     // tiles of one tile-column share their B (weights) in L2
  n_blk = tile / g.tiles_m;
}

}  // namespace streamk_detail

template <class KT>
__global__ void __launch_bounds__(KT::NumThreads, 1)
    nvfp4_gemm_1sm_streamk_kernel(const __grid_constant__ Nvfp4StreamKParams ps) {
#if defined(BLACKHOLE_ARCH_SM100)
  using namespace ptx;
  using namespace streamk_detail;
  using skinny_detail::ld_acquire;
  using skinny_detail::st_release;
  constexpr int S = KT::Stages;
  const Nvfp4GemmParams& p = ps.g;

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
  volatile uint32_t* const ticket_slot = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);
  volatile uint32_t* const gen_slot = reinterpret_cast<volatile uint32_t*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // Start order and launch tag, as in the skinny schedule: the generation is read before the
    // ticket is taken and advanced by the last taker after its reset.
    const uint32_t gen = ld_acquire(ps.ticket + 1);
    __threadfence();
    const uint32_t t = atomicAdd(ps.ticket, 1u);
    if (t == uint32_t(ps.grid) - 1u) {
      atomicExch(ps.ticket, 0u);
      __threadfence();
      atomicExch(ps.ticket + 1, gen + 1u);
      __threadfence();
    }
    *ticket_slot = t;
    *gen_slot = (gen << 1) | 1u;
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
  const int c = static_cast<int>(*ticket_slot);
  const uint32_t tag = *gen_slot;
  pdl_launch_dependents();  // every CTA of this launch has its ticket: the next may start
  // the previous kernel in the stream must be complete before global memory is touched
  pdl_wait_prior_grid();

  if (warp == KT::ProducerWarp) {
    // ------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();
      const uint64_t pol_b = l2_policy_evict_first();   // the weights stream once
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      Walk w = walk(ps, c);
      Segment sg;
      while (ok && w.next(sg)) {
        int m_blk, n_blk;
        tile_mn(p, sg.tile, m_blk, n_blk);
        const bool sfb_hi = (2 * n_blk + 1) < p.n_blocks128;
        const uint32_t bytes =
            KT::ATx + KT::BTx + KT::SFABytes +
            ((sfb_hi || p.sf_tail) ? KT::SFBBytes : KT::SFBBytes / 2);
        const uint8_t* sfa_src = p.sfa + (int64_t(m_blk) * p.sf_k_atoms) * 512;
        const uint8_t* sfb_src0 = p.sfb + (int64_t(2 * n_blk) * p.sf_k_atoms) * 512;
        const uint8_t* sfb_src1 = sfb_src0 + int64_t(p.sf_k_atoms) * 512;
        for (int kt = sg.kt0; kt < sg.kt1; ++kt) {
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
        // let the copies already in flight land before the CTA goes away
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
    constexpr uint32_t idesc = idesc_block_scaled(KT::TileM, KT::TileN, KT::Fmt::AFormat,
                                                  KT::Fmt::BFormat, KT::Fmt::ScaleType);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    bool issued_any = false;
    auto copy_sf = [&](int st) {
      const uint32_t sfa_s = sSFA + st * KT::SFABytes;
      const uint32_t sfb_s = sSFB + st * KT::SFBBytes;
      const uint32_t ta = tmem + KT::SfCol;
#pragma unroll
      for (int j = 0; j < KT::SfAtoms; ++j) {
        tc_cp_32x128b_warpx4_w(ta + 4 * j, desc_sf_atom(sfa_s + 512 * j));
        tc_cp_32x128b_warpx4_w(ta + 4 * KT::SfAtoms + 8 * j, desc_sf_atom(sfb_s + 512 * j));
        tc_cp_32x128b_warpx4_w(ta + 4 * KT::SfAtoms + 8 * j + 4,
                               desc_sf_atom(sfb_s + KT::SFBBytes / 2 + 512 * j));
      }
    };
    Walk w = walk(ps, c);
    Segment sg;
    while (ok && w.next(sg)) {
      if (!wait_bounded_warp(acc_empty, acc_phase ^ 1u, abort_flag, p.status, kStatusMmaTimeout)) {
        ok = false;
        break;
      }
      tc_fence_after();
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
        copy_sf(stage);
        const uint64_t adesc = desc_kmajor<KT::RowBytes>(sA + stage * KT::ABytes);
        const uint64_t bdesc = desc_kmajor<KT::RowBytes>(sB + stage * KT::BBytes);
        const uint32_t ta = tmem + KT::SfCol;
#pragma unroll
        for (int j = 0; j < KT::KSteps; ++j) {
          const int at = j / KT::StepsPerAtom;
          const uint32_t sid = KT::Geo::sf_id(j);
          tc_mma_bs_w<typename KT::Fmt>(
              tmem + KT::AccCol, adesc + 2 * j, bdesc + 2 * j, idesc_with_sf_id(idesc, sid),
              sf_tmem_addr(ta + 4 * at, sid), sf_tmem_addr(ta + 4 * KT::SfAtoms + 8 * at, sid),
              (kt != sg.kt0 || j != 0) ? 1u : 0u);
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
      tc_commit_w(drain_bar);
      detail::drain_wait(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ----------------------------------------
    const int q = warp & 3;                                   // TMEM lane quadrant
    const int half = (warp - KT::FirstEpiWarp) >> 2;          // column half of the tile
    const int fi = q + 4 * half;                              // this warp's flag slot
    const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * q) << 16) + KT::AccCol + 128 * half;
    // this warp's 32 rows x 128 columns of a partial slot, as 32 lines of 512 bytes (4 columns
    // of the 32 rows each); lane i holds row 32q + i
    auto part_of = [&](int cta) {
      return ps.ws + ((int64_t(cta) * 2 + half) * 4 + q) * (32 * 128) + lane * 4;
    };
    uint32_t acc_phase = 0;
    Walk w = walk(ps, c);
    Segment sg;
    while (w.next(sg)) {
      int m_blk, n_blk;
      tile_mn(p, sg.tile, m_blk, n_blk);
      if (!wait_bounded_warp(acc_full, acc_phase, abort_flag, p.status, kStatusEpilogueTimeout)) break;
      tc_fence_after();
      uint32_t v[4][32];
      tmem_ld_32x32b_x32(t_row + 0, v[0]);
      tmem_ld_32x32b_x32(t_row + 32, v[1]);
      tmem_ld_32x32b_x32(t_row + 64, v[2]);
      tmem_ld_32x32b_x32(t_row + 96, v[3]);
      tmem_ld_wait();
      reg_fence(v[0]);
      reg_fence(v[1]);
      reg_fence(v[2]);
      reg_fence(v[3]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      acc_phase ^= 1u;

      const int row0 = m_blk * KT::TileM + 32 * q;
      const bool row_live = row0 + lane < p.M;
      const bool finisher = sg.kt1 == p.k_tiles;
      if (!finisher) {
        // Partial of a tile finished by a later CTA: park it, then raise this warp's flag.
        float* dst = part_of(c);
        if (row_live) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const uint32_t (&r)[32] = v[j >> 3];
            const int i = (j & 7) * 4;
            __stcg(reinterpret_cast<float4*>(dst + j * 128),
                   make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                               __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])));
          }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release(ps.flags + kSkinnyFlagsPerCta * c + fi, tag);
        continue;
      }
      if (sg.kt0 > 0) {
        // Add the partials of the earlier CTAs sharing this tile, nearest first (a fixed
        // order: the result does not depend on timing).
        const int64_t t0 = int64_t(sg.tile) * p.k_tiles;
        bool ok = true;
        for (int cc = c - 1; cc >= 0 && range_start(ps, cc + 1) > t0; --cc) {
          uint32_t* flag = ps.flags + kSkinnyFlagsPerCta * cc + fi;
          int ready = 1;
          if (lane == 0) {
            const uint64_t tw = globaltimer_ns();
            while (ld_acquire(flag) != tag) {
              if (*abort_flag) { ready = 0; break; }
              if (globaltimer_ns() - tw > ps.partial_wait_ns) {
                *abort_flag = 1;
                if (p.status) atomicOr(p.status, kStatusEpilogueTimeout);
                ready = 0;
                break;
              }
            }
          }
          ready = __shfl_sync(0xFFFFFFFFu, ready, 0);
          if (!ready) {
            ok = false;
            break;
          }
          (void)ld_acquire(flag);
          const float* src = part_of(cc);
          if (row_live) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              uint32_t (&r)[32] = v[j >> 3];
              const int i = (j & 7) * 4;
              const float4 a = __ldcg(reinterpret_cast<const float4*>(src + j * 128));
              r[i] = __float_as_uint(__uint_as_float(r[i]) + a.x);
              r[i + 1] = __float_as_uint(__uint_as_float(r[i + 1]) + a.y);
              r[i + 2] = __float_as_uint(__uint_as_float(r[i + 2]) + a.z);
              r[i + 3] = __float_as_uint(__uint_as_float(r[i + 3]) + a.w);
            }
          }
          __syncwarp();
          if (lane == 0) st_release(flag, 0u);
        }
        if (!ok) break;
      }

      // alpha * acc -> BF16 -> this warp's 1 KB staging box -> TMA store, 16 columns at a
      // time (the one-SM schedule's epilogue).
      const int col0 = n_blk * KT::TileN + 128 * half;
      const uint32_t box = sStage + (warp - KT::FirstEpiWarp) * KT::StoreBoxBytes;
      const uint32_t my_row = box + lane * 32;
      const uint32_t sw = (lane >> 2) & 1;
      const float a = p.alpha;
      const bool live = row0 < p.M && col0 < p.N;
      const uint64_t pol_d = l2_policy_evict_first();
#pragma unroll
      for (int g = 0; g < 4; ++g) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (lane == 0) bulk_wait_group_read<0>();   // previous box has been read out
          __syncwarp();
#pragma unroll
          for (int cc2 = 0; cc2 < 2; ++cc2) {
            const int i = 16 * h + 8 * cc2;
            const uint32_t (&r)[32] = v[g];
            st_shared_v4(my_row + ((cc2 ^ sw) << 4),
                         detail::pack_bf16x2(a * __uint_as_float(r[i + 0]), a * __uint_as_float(r[i + 1])),
                         detail::pack_bf16x2(a * __uint_as_float(r[i + 2]), a * __uint_as_float(r[i + 3])),
                         detail::pack_bf16x2(a * __uint_as_float(r[i + 4]), a * __uint_as_float(r[i + 5])),
                         detail::pack_bf16x2(a * __uint_as_float(r[i + 6]), a * __uint_as_float(r[i + 7])));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && live && col0 + 32 * g + 16 * h < p.N) {
            tma_store_2d(&p.tmap_d, box, col0 + 32 * g + 16 * h, row0, pol_d);
            bulk_commit_group();
          }
        }
      }
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
inline cudaError_t launch_1sm_streamk(int M, int N, int K, const void* A, const void* SFA,
                                      const void* B, const void* SFB, void* D, float alpha,
                                      void* ws, int64_t ws_bytes, DeviceState* st, int dev,
                                      cudaStream_t stream,
                                      uint64_t partial_wait_ns = ptx::kWaitLimitNs) {
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255u)) return cudaErrorInvalidValue;
  if (nvfp4_1sm_streamk_workspace_bytes(st->num_sms) > ws_bytes) return cudaErrorInvalidValue;
  cudaError_t e = set_smem_once(nvfp4_gemm_1sm_streamk_kernel<KT>, KT::SmemBytes, dev);
  if (e != cudaSuccess) return e;
  Nvfp4StreamKParams ps;
  Nvfp4GemmParams& p = ps.g;
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
  ps.units = int64_t(p.num_tiles) * p.k_tiles;
  int grid = st->num_sms;
  if (ps.units < grid) grid = static_cast<int>(ps.units);
  ps.grid = grid;
  ps.flags = static_cast<uint32_t*>(ws);
  ps.ticket = ps.flags + kSkinnyFlagsPerCta * st->num_sms;
  ps.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + nvfp4_skinny_flag_bytes(st->num_sms));
  ps.partial_wait_ns = partial_wait_ns;
  e = launch_pdl(nvfp4_gemm_1sm_streamk_kernel<KT>, dim3(grid), dim3(KT::NumThreads),
                 KT::SmemBytes, stream, ps);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace detail

#endif  // __CUDACC__

}  // namespace blackhole::sm100
