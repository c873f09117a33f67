#pragma once

// =====================================================================================
// blackhole / sm100 / NVFP4 (E2M1 + UE4M3 per-16 block scale) x NVFP4 -> BF16 GEMM
// -------------------------------------------------------------------------------------
// D = bf16(alpha * A . B^T) on B200 (sm_100a), hand-written tcgen05 / TMA PTX:
//
//   * A: M x K E2M1, K-contiguous, two values per byte (even k in the low nibble)
//   * B: N x K E2M1, K-contiguous
//   * SFA / SFB: UE4M3, one per 16 K-elements, 128x4 blocked layout
//     (blackhole/common/sf_layout.hpp; the reference's make_layout_SFA/SFB)
//   * D: M x N BF16 row-major; FP32 accumulation in tensor memory (TMEM)
//
// Same operator call as the reference's sm_120 kernel
// (include/blackhole/sm120/nvfp4_gemm.hpp:588-637), plus an alpha (global scale) overload.
//
// Schedules (chosen by shape):
//   * M <= 16 : skinny schedule (nvfp4_gemm_skinny.hpp) -- swap-AB, stream-K over all SMs,
//                HBM-bound; needs a small FP32 workspace (allocated here per device and
//                stream on first use, or passed by the caller: nvfp4_bf16_gemm_ex).  It warms
//                L2 with its first B / SFB tiles while the previous kernel in the stream is
//                finishing (a prefetch only: results are those of plain stream order);
//   * 16 < M <= 256 : one-SM schedule (nvfp4_gemm_1sm.hpp) -- 128 x 256 tiles.  Measured on
//                B200 (K = 1024..16384, N = 2048..28672): faster than the skinny schedule in
//                every case but one from M = 32 up (M = 128, N = 28672, K = 8192: 30.5 vs
//                38.3 us; M = 128, N = 4096, K = 4096: 10.8 vs 31.9 us), slower at M = 16
//                (25.2 vs 30.9 us at N = 28672);
//   * M > 256  : two-SM schedule (nvfp4_gemm_2sm.hpp) -- 256 x 256 tiles per CTA pair
//                (cta_group::2): a third less operand traffic into each SM than the one-SM
//                tile, which on B200 is what limits the tensor pipe once the kernel is power
//                capped (measured at 8192^3 with N(0,1) data: 220.8 us vs 226.5 us per launch).
//
// Shapes: M >= 1, N % 8 == 0, K % 32 == 0.  The reference requires M % 128 == 0,
// N % 128 == 0 and K % 256 == 0 (nvfp4_gemm.hpp:594).  With a K tail, the scale factors of
// the K-groups past K (padding of the last 128x4 atom) must be finite: they multiply zeros.  Every mbarrier wait in the kernels is
// bounded: a stalled pipeline records a status bit (blackhole_sm100_device_status) and returns.
// =====================================================================================

#include <cstddef>
#include <cstdint>

#include <cuda_runtime_api.h>

#include <blackhole/common/arch.hpp>
#include <blackhole/common/sf_layout.hpp>
#include <blackhole_sm100.h>

#include <blackhole/sm100/nvfp4_gemm_common.hpp>

#if defined(__CUDACC__)
#include <map>
#include <utility>

#include <blackhole/sm100/nvfp4_gemm_1sm.hpp>
#include <blackhole/sm100/nvfp4_gemm_2sm.hpp>
#include <blackhole/sm100/nvfp4_gemm_skinny.hpp>
#endif

namespace blackhole::sm100 {

// kSkinnyNoPrefetch is the skinny schedule without the L2 prefetch of B / SFB that it issues
// while the previous kernel in the stream is finishing (same results; for measurement).
enum class Nvfp4Schedule : int { kAuto = 0, kOneSm = 1, kTwoSm = 2, kSkinny = 3, kSkinnyNoPrefetch = 4 };

#if defined(__CUDACC__)

namespace detail {

// Workspace of the skinny schedule owned by the library: one per (device, stream), grown
// on demand, flag words zeroed at allocation.  Calls on the same stream are ordered, so
// they may share it; different streams get different buffers.
inline cudaError_t library_workspace(int dev, cudaStream_t stream, int64_t bytes, void** out) {
  struct Ws {
    void* ptr = nullptr;
    int64_t bytes = 0;
  };
  static std::mutex mu;
  static std::map<std::pair<int, uintptr_t>, Ws> pool;
  std::lock_guard<std::mutex> lock(mu);
  Ws& w = pool[{dev, reinterpret_cast<uintptr_t>(stream)}];
  if (w.bytes < bytes) {
    if (w.ptr) {
      cudaError_t e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) return e;
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    cudaError_t e = cudaMalloc(&w.ptr, static_cast<size_t>(bytes));
    if (e != cudaSuccess) return e;
    e = cudaMemset(w.ptr, 0, static_cast<size_t>(bytes));
    if (e != cudaSuccess) return e;
    w.bytes = bytes;
  }
  *out = w.ptr;
  return cudaSuccess;
}

}  // namespace detail

// Full control: element format, schedule choice and (for the skinny schedule) a caller-owned
// workspace.  workspace == nullptr selects the library-owned workspace.
template <class Fmt>
inline cudaError_t block_scaled_bf16_gemm_ex(int M, int N, int K, void const* A, void const* SFA,
                                             void const* B, void const* SFB, void* D, float alpha,
                                             Nvfp4Schedule schedule, void* workspace,
                                             int64_t workspace_bytes, cudaStream_t stream) {
  cudaError_t e = nvfp4_check_args(M, N, K, A, SFA, B, SFB, D);
  if (e != cudaSuccess) return e;
  e = detail::format_check_args<Fmt>(K, B);
  if (e != cudaSuccess) return e;
  detail::DeviceState* st = detail::prepare_device();
  if (!st) return cudaErrorInvalidDevice;
  if (st->init_err != cudaSuccess) return st->init_err;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (schedule == Nvfp4Schedule::kAuto)
    schedule = M <= 16    ? Nvfp4Schedule::kSkinny
               : M <= 256 ? Nvfp4Schedule::kOneSm
                          : Nvfp4Schedule::kTwoSm;
  switch (schedule) {
    case Nvfp4Schedule::kOneSm:
      return detail::launch_1sm<Nvfp4GemmTraitsT<4, Fmt>>(M, N, K, A, SFA, B, SFB, D, alpha, st,
                                                           dev, stream);
    case Nvfp4Schedule::kTwoSm:
      return detail::launch_2sm<Nvfp4Gemm2SmTraitsT<5, Fmt>>(M, N, K, A, SFA, B, SFB, D, alpha,
                                                              st, dev, stream);
    case Nvfp4Schedule::kSkinny:
    case Nvfp4Schedule::kSkinnyNoPrefetch: {
      if (M > 128) return cudaErrorInvalidValue;
      const int64_t need = nvfp4_skinny_workspace_bytes(st->num_sms, nvfp4_skinny_mpad(M));
      if (!workspace) {
        e = detail::library_workspace(dev, stream, need, &workspace);
        if (e != cudaSuccess) return e;
        workspace_bytes = need;
      }
      return block_scaled_bf16_gemm_skinny<Fmt>(M, N, K, A, SFA, B, SFB, D, alpha, workspace,
                                                workspace_bytes, stream, 1 << 30,
                                                schedule == Nvfp4Schedule::kSkinny);
    }
    default:
      return cudaErrorInvalidValue;
  }
}

inline cudaError_t nvfp4_bf16_gemm_ex(int M, int N, int K, void const* A, void const* SFA,
                                      void const* B, void const* SFB, void* D, float alpha,
                                      Nvfp4Schedule schedule, void* workspace,
                                      int64_t workspace_bytes, cudaStream_t stream) {
  return block_scaled_bf16_gemm_ex<Nvfp4Format>(M, N, K, A, SFA, B, SFB, D, alpha, schedule,
                                                workspace, workspace_bytes, stream);
}

// MXFP4 (OCP MX: E2M1 elements, one UE8M0 scale per 32 along K, same 128x4 layout with
// 32-element groups: sf_storage_bytes_vs(MN, K, 32) bytes); not in the reference, served by
// the same schedules.  Shapes as nvfp4_bf16_gemm.
inline cudaError_t mxfp4_bf16_gemm_ex(int M, int N, int K, void const* A, void const* SFA,
                                      void const* B, void const* SFB, void* D, float alpha,
                                      Nvfp4Schedule schedule, void* workspace,
                                      int64_t workspace_bytes, cudaStream_t stream) {
  return block_scaled_bf16_gemm_ex<Mxfp4Format>(M, N, K, A, SFA, B, SFB, D, alpha, schedule,
                                                workspace, workspace_bytes, stream);
}
// MXFP8 x MXFP4: A (M x K) is E4M3, one byte per element, with UE8M0 scales per 32; B (N x K)
// is packed E2M1 (MXFP4); both scale tensors in the 128x4 layout with 32-element groups.
// tcgen05.mma kind::mxf8f6f4 (half the FP4 rate).  Shapes as nvfp4_bf16_gemm plus
// K % 128 == 0 and B 32-byte aligned.
inline cudaError_t mxf8f4_bf16_gemm_ex(int M, int N, int K, void const* A, void const* SFA,
                                       void const* B, void const* SFB, void* D, float alpha,
                                       Nvfp4Schedule schedule, void* workspace,
                                       int64_t workspace_bytes, cudaStream_t stream) {
  return block_scaled_bf16_gemm_ex<Mxf8f4Format>(M, N, K, A, SFA, B, SFB, D, alpha, schedule,
                                                 workspace, workspace_bytes, stream);
}
inline cudaError_t mxfp4_bf16_gemm(int M, int N, int K, void const* A, void const* SFA,
                                   void const* B, void const* SFB, void* D, float alpha = 1.0f,
                                   cudaStream_t stream = nullptr) {
  return mxfp4_bf16_gemm_ex(M, N, K, A, SFA, B, SFB, D, alpha, Nvfp4Schedule::kAuto, nullptr, 0,
                            stream);
}

// GEMM with the output gathered in the same kernel: the M x N result goes to columns
// [col0, col0 + N) of each of the ndst row-major BF16 buffers dst[0..ndst) (rows ldd
// elements apart).  dst[0] is this GPU's buffer; the others are typically other GPUs' buffers
// mapped into this process (CUDA IPC), written tile by tile with plain stores over NVLink
// while the next tiles are computed.  Used by the N-split: rank r of P passes every rank's
// buffer and col0 = r * N, so each GPU ends with the whole row-major M x (P*N) result.  The
// call orders nothing across GPUs: the caller synchronises the ranks after it (and before
// reusing a buffer another rank still reads).  M <= 128 runs the skinny schedule (its
// epilogue stores 2-byte elements to every buffer), larger M the two-SM schedule.
inline cudaError_t nvfp4_bf16_gemm_gather(int M, int N, int K, void const* A, void const* SFA,
                                          void const* B, void const* SFB, void* const* dst,
                                          int ndst, int64_t col0, int64_t ldd, float alpha,
                                          cudaStream_t stream = nullptr) {
  if (!dst || ndst < 1 || ndst > kMaxGatherPeers + 1) return cudaErrorInvalidValue;
  cudaError_t e = nvfp4_check_args(M, N, K, A, SFA, B, SFB, dst[0]);
  if (e != cudaSuccess) return e;
  for (int i = 0; i < ndst; ++i)
    if (!dst[i] || (reinterpret_cast<uintptr_t>(dst[i]) & 15u)) return cudaErrorInvalidValue;
  if (col0 < 0 || col0 % 8 != 0 || ldd % 8 != 0 || col0 + N > ldd) return cudaErrorInvalidValue;
  if (static_cast<int64_t>(M) * ldd > (int64_t(1) << 46)) return cudaErrorInvalidValue;
  detail::DeviceState* st = detail::prepare_device();
  if (!st) return cudaErrorInvalidDevice;
  if (st->init_err != cudaSuccess) return st->init_err;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const detail::GatherSpec g{dst, ndst, col0, ldd};
  if (M <= 128) {   // decode-sized: the skinny schedule, its epilogue storing to every buffer
    const int64_t need = nvfp4_skinny_workspace_bytes(st->num_sms, nvfp4_skinny_mpad(M));
    void* ws = nullptr;
    e = detail::library_workspace(dev, stream, need, &ws);
    if (e != cudaSuccess) return e;
    return block_scaled_bf16_gemm_skinny<Nvfp4Format>(M, N, K, A, SFA, B, SFB, dst[0], alpha, ws,
                                                      need, stream, 1 << 30, true, &g);
  }
  return detail::launch_2sm<Nvfp4Gemm2SmTraitsT<5, Nvfp4Format>>(
      M, N, K, A, SFA, B, SFB, dst[0], alpha, st, dev, stream, &g);
}

//   A_packed : E2M1, M x K, K-contiguous (two per byte, low nibble first)
//   SFA      : UE4M3 in the 128x4 layout (make_layout_SFA(M, K)), sf_storage_bytes(M, K) bytes
//   B_packed : E2M1, N x K, K-contiguous
//   SFB      : UE4M3 in the 128x4 layout, sf_storage_bytes(N, K) bytes
//   D        : BF16, M x N row-major;  D = bf16(alpha * sum_k a*sfa * b*sfb)
inline cudaError_t nvfp4_bf16_gemm(int M, int N, int K, void const* A_packed, void const* SFA,
                                   void const* B_packed, void const* SFB, void* D, float alpha,
                                   cudaStream_t stream = nullptr) {
  return nvfp4_bf16_gemm_ex(M, N, K, A_packed, SFA, B_packed, SFB, D, alpha, Nvfp4Schedule::kAuto,
                            nullptr, 0, stream);
}

// The reference's exact nine-argument call (alpha = 1).
inline cudaError_t nvfp4_bf16_gemm(int M, int N, int K, void const* A_packed, void const* SFA,
                                   void const* B_packed, void const* SFB, void* D,
                                   cudaStream_t stream = nullptr) {
  return nvfp4_bf16_gemm(M, N, K, A_packed, SFA, B_packed, SFB, D, 1.0f, stream);
}

#else  // !__CUDACC__: host-compiler users reach the same operator through the C ABI.

inline cudaError_t nvfp4_bf16_gemm(int M, int N, int K, void const* A_packed, void const* SFA,
                                   void const* B_packed, void const* SFB, void* D, float alpha,
                                   cudaStream_t stream = nullptr) {
  return static_cast<cudaError_t>(
      blackhole_sm100_nvfp4_bf16_gemm(M, N, K, A_packed, SFA, B_packed, SFB, D, alpha, stream));
}
inline cudaError_t nvfp4_bf16_gemm(int M, int N, int K, void const* A_packed, void const* SFA,
                                   void const* B_packed, void const* SFB, void* D,
                                   cudaStream_t stream = nullptr) {
  return nvfp4_bf16_gemm(M, N, K, A_packed, SFA, B_packed, SFB, D, 1.0f, stream);
}

#endif  // __CUDACC__

}  // namespace blackhole::sm100
