#pragma once

// Stream-ordered barrier across the GPUs of a gathered N-split (nvfp4_bf16_gemm_gather).
//
// Every rank owns an array of `world` 64-bit flag words, zero at first and mapped into every
// other rank's process.  A barrier with epoch e (1, 2, 3, ... per call) stores e, with a
// system-scope release, into this rank's word of every peer's array -- after everything
// earlier in the stream, the gather kernels' stores into the peers' buffers included -- and
// then waits until every peer's word in its own array has reached e (system-scope acquire).
// Kernels after it in the stream therefore see every rank's tiles.  It replaces a one-element
// NCCL all-reduce (~25 us on two B200s) with one small kernel per rank and one NVLink store
// per peer.  The wait is bounded: past limit_ns it sets kStatusBarrierTimeout in the device
// status word and returns, so a rank that never arrives surfaces as an error instead of a
// hang.  One barrier per GPU: the ranks' barriers wait on one another, so they must run on
// different GPUs, never as several launches on one GPU.

#include <blackhole/sm100/nvfp4_gemm_common.hpp>

namespace blackhole::sm100 {

#if defined(__CUDACC__)

namespace barrier_detail {

struct PeerFlags {
  uint64_t* f[kMaxGatherPeers + 1];   // rank q's flag array as mapped in this process
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One warp: lane q signals peer q, then waits for peer q's signal.
__global__ void peer_barrier_kernel(PeerFlags flags, int world, int rank, uint64_t epoch,
                                    uint64_t limit_ns, uint32_t* status) {
  const int q = static_cast<int>(threadIdx.x);
  if (q >= world || q == rank) return;
  st_release_sys(flags.f[q] + rank, epoch);
  const uint64_t* mine = flags.f[rank] + q;
  const uint64_t t0 = ptx::globaltimer_ns();
  while (ld_acquire_sys(mine) < epoch) {
    if (ptx::globaltimer_ns() - t0 > limit_ns) {
      atomicOr(status, kStatusBarrierTimeout);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace barrier_detail

// flags[q]: rank q's flag array (world 64-bit words, 8-byte aligned) as mapped in this
// process, flags[rank] this GPU's own; epoch >= 1, one more than the previous call's;
// 0 < limit_ns <= 10 s.  world == 1 launches nothing.
inline cudaError_t peer_barrier(void* const* flags, int world, int rank, uint64_t epoch,
                                uint64_t limit_ns, cudaStream_t stream = nullptr) {
  if (!flags || world < 1 || world > kMaxGatherPeers + 1 || rank < 0 || rank >= world ||
      epoch < 1 || limit_ns == 0 || limit_ns > 10000000000ull)
    return cudaErrorInvalidValue;
  barrier_detail::PeerFlags f{};
  for (int q = 0; q < world; ++q) {
    if (!flags[q] || (reinterpret_cast<uintptr_t>(flags[q]) & 7u)) return cudaErrorInvalidValue;
    f.f[q] = static_cast<uint64_t*>(flags[q]);
  }
  if (world == 1) return cudaSuccess;
  detail::DeviceState* st = detail::prepare_device();
  if (!st) return cudaErrorInvalidDevice;
  if (st->init_err != cudaSuccess) return st->init_err;
  barrier_detail::peer_barrier_kernel<<<1, 32, 0, stream>>>(f, world, rank, epoch, limit_ns,
                                                             st->status);
  return cudaGetLastError();
}

#endif  // __CUDACC__

}  // namespace blackhole::sm100
