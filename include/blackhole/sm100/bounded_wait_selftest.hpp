#pragma once

// Self-test of the bounded-wait / abort protocol that every GEMM schedule uses, without
// faulting or hanging the GPU.  One CTA of two warps plays the two sides of a pipeline whose
// partner never shows up:
//
//   * warp 0 ("producer") waits with wait_bounded on an mbarrier that nothing arrives on;
//     after `limit_ns` it gives up, raises the CTA abort flag and or-s kStatusLoadTimeout
//     into the module status word;
//   * warp 1 ("consumer") holds 32 TMEM columns and waits warp-uniformly (wait_bounded_warp)
//     on another barrier that nothing arrives on, with a limit 4x longer; it must leave
//     because of the abort flag, not its own limit, so kStatusMmaTimeout stays clear;
//   * both warps meet at a __syncthreads and warp 1 frees its TMEM, as the GEMM kernels do
//     on their abort path.
//
// result[0..1] = 1 if warp 0 / warp 1 saw its wait complete (expected 0, 0);
// result[2..3] = nanoseconds warp 0 / warp 1 spent waiting.
// The wait always ends within limit_ns (warp 0) plus one polling interval (warp 1), so the
// kernel terminates on its own.

#include <cstdint>

#include <cuda_runtime_api.h>

#include <blackhole/common/arch.hpp>
#include <blackhole/sm100/nvfp4_gemm_common.hpp>
#include <blackhole/sm100/ptx.hpp>

namespace blackhole::sm100 {
namespace detail {

__global__ void __launch_bounds__(64, 1)
    bounded_wait_selftest_kernel(uint32_t* status, uint64_t limit_ns, uint64_t* result) {
#if defined(BLACKHOLE_ARCH_SM100)
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t bar_free = ptx::smem_u32(&bars[0]);
  const uint32_t bar_full = ptx::smem_u32(&bars[1]);
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_free, 1);
    ptx::mbar_init(bar_full, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(&tmem_slot), 32);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  const uint64_t t0 = ptx::globaltimer_ns();
  bool done = false;
  if (warp == 0) {
    if (lane == 0)
      done = ptx::wait_bounded(bar_free, 0, &abort_flag, status, kStatusLoadTimeout, limit_ns);
    __syncwarp();
  } else {
    done = ptx::wait_bounded_warp(bar_full, 0, &abort_flag, status, kStatusMmaTimeout,
                                  4 * limit_ns);
  }
  const uint64_t t1 = ptx::globaltimer_ns();
  if (lane == 0) {
    result[warp] = done ? 1u : 0u;
    result[2 + warp] = t1 - t0;
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem_slot, 32);
#endif
}

}  // namespace detail

// Launches the self-test on `stream`; result must hold 4 device uint64 words.
inline cudaError_t bounded_wait_selftest(uint64_t limit_ns, uint64_t* result,
                                         cudaStream_t stream) {
  if (!result || limit_ns == 0 || limit_ns > 2000000000ull) return cudaErrorInvalidValue;
  detail::DeviceState* st = detail::prepare_device();
  if (!st) return cudaErrorInvalidDevice;
  if (st->init_err != cudaSuccess) return st->init_err;
  detail::bounded_wait_selftest_kernel<<<1, 64, 0, stream>>>(st->status, limit_ns, result);
  return cudaGetLastError();
}

}  // namespace blackhole::sm100
