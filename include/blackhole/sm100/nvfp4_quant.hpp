#pragma once

// =====================================================================================
// blackhole / sm100 / NVFP4 quantiser: FP32 or BF16 (rows x K) -> packed E2M1 + UE4M3
// per-16 scale factors in the 128x4 layout + one FP32 global scale.
// -------------------------------------------------------------------------------------
// Recipe (per tensor X):
//   amax = max |X|;                 g = amax / (448 * 6)
//   per 16-element block b:         s_b = UE4M3_rne((amax_b / 6) / g)
//   per element:                    q = E2M1_rne(x / (s_b * g))   (q = 0 when s_b == 0)
// A GEMM of two such tensors uses alpha = gA * gB.  Each step is one IEEE-rounded FP32
// operation, in this order, so the result is bit-reproducible on the host.
//
// This is the step before the GEMM that the reference performs on the host with CUTLASS
// converters (example/nvfp4_bf16_gemm.cu:60-71, :104-133).  Two HBM-bound kernels:
// a grid-stride amax reduction, then one thread per 16-element block.
// =====================================================================================

#include <algorithm>
#include <cstdint>

#include <cuda_runtime_api.h>

#include <blackhole/common/sf_layout.hpp>

#if defined(__CUDACC__)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#endif

namespace blackhole::sm100 {

#if defined(__CUDACC__)

namespace quant_detail {

// E2M1, round to nearest even, saturating; sign kept.  Magnitudes by code:
// 0, 0.5, 1, 1.5, 2, 3, 4, 6; a midpoint goes to the code whose last bit is 0.
__device__ __forceinline__ uint32_t e2m1_rne(float x) {
  const uint32_t sign = (__float_as_uint(x) >> 28) & 8u;
  const float a = fabsf(x);
  uint32_t m;
  if (a <= 0.25f) m = 0;
  else if (a < 0.75f) m = 1;
  else if (a <= 1.25f) m = 2;
  else if (a < 1.75f) m = 3;
  else if (a <= 2.5f) m = 4;
  else if (a < 3.5f) m = 5;
  else if (a <= 5.0f) m = 6;
  else m = 7;                       // above 5 (and NaN, which fails every test) -> 6
  return sign | m;
}

__device__ __forceinline__ float ue4m3_value(uint32_t code) {
  const uint32_t e = (code >> 3) & 15u, m = code & 7u;
  if (e == 0) return static_cast<float>(m) * 0.001953125f;                 // m * 2^-9
  return __uint_as_float(((e + 120u) << 23) | (m << 20));                  // (1+m/8)*2^(e-7)
}

// Unsigned E4M3 of |v|: bias 7, 3 mantissa bits, subnormal step 2^-9, saturates to 448.
__device__ __forceinline__ uint32_t ue4m3_rne(float v) {
  const uint32_t u = __float_as_uint(v) & 0x7FFFFFFFu;
  if (u > 0x7F800000u) return 0x7Fu;                 // NaN
  if (u >= 0x43E00000u) return 0x7Eu;                // >= 448 (inf included)
  const int exp = static_cast<int>(u >> 23) - 127;
  if (exp < -6) {                                    // below 2^-6: multiples of 2^-9
    return static_cast<uint32_t>(__float2int_rn(__uint_as_float(u) * 512.0f));
  }
  uint32_t e = static_cast<uint32_t>(exp + 7);
  uint32_t keep = (u >> 20) & 7u;
  const uint32_t rest = u & 0xFFFFFu;
  if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) ++keep;
  if (keep == 8u) { keep = 0; ++e; }
  uint32_t code = (e << 3) | keep;
  return code >= 0x7Fu ? 0x7Eu : code;
}

// 16 consecutive elements -> registers (vectorised loads).
__device__ __forceinline__ void load16(const float* p, float (&x)[16]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 v = __ldcs(q + i);
    x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
  }
}
__device__ __forceinline__ void load16(const __nv_bfloat16* p, float (&x)[16]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint4 v = __ldcs(q + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
      x[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

template <class T>
__global__ void __launch_bounds__(256) amax_kernel(const T* __restrict__ x, int64_t n_blocks16,
                                                   float* __restrict__ scales) {
  float m = 0.0f;
  for (int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; b < n_blocks16;
       b += int64_t(gridDim.x) * blockDim.x) {
    float v[16];
    load16(x + b * 16, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    // non-negative floats order like their bit patterns
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(scales), __float_as_uint(m));
  }
}

// One thread per (row, 16-element group) over the layout's padded extent: rows padded to
// 128 and groups to a multiple of 4; padding entries get s = 0.
template <class T>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ x, int rows, int K,
                                                       uint8_t* __restrict__ packed,
                                                       uint8_t* __restrict__ sf,
                                                       float* __restrict__ scales) {
  const int groups = K / 16;
  const int groups_pad = (groups + 3) / 4 * 4;
  const int64_t rows_pad = (int64_t(rows) + 127) / 128 * 128;
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (idx >= rows_pad * groups_pad) return;
  const int64_t r = idx / groups_pad;
  const int64_t kg = idx - r * groups_pad;
  const float amax = scales[0];
  const float g = amax / 2688.0f;
  if (idx == 0) scales[1] = g;
  uint32_t s_code = 0;
  if (r < rows && kg < groups) {
    float v[16];
    load16(x + r * K + kg * 16, v);
    float amax_b = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax_b = fmaxf(amax_b, fabsf(v[i]));
    float s_val = 0.0f;
    if (g > 0.0f) {
      s_code = ue4m3_rne((amax_b / 6.0f) / g);
      s_val = ue4m3_value(s_code);
    }
    const float scale = s_val * g;
    uint32_t lo = 0, hi = 0;
    if (s_val != 0.0f) {
#pragma unroll
      for (int i = 0; i < 8; ++i) lo |= e2m1_rne(v[i] / scale) << (4 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) hi |= e2m1_rne(v[8 + i] / scale) << (4 * i);
    }
    *reinterpret_cast<uint2*>(packed + (r * K + kg * 16) / 2) = make_uint2(lo, hi);
  }
  sf[blackhole::sf_offset(r, kg, K)] = static_cast<uint8_t>(s_code);
}

// MXFP4 (OCP MX v1.0): one thread per (row, 32-element group) over the padded extent.
// Shared exponent e = floor(log2(amax_b)) - 2, read from amax_b's exponent bits (zero and
// subnormal amax -> -127), clamped to [-127, 127]; scale code e + 127; element codes
// e2m1(x * 2^-e) with the power of two built exactly.  Padding entries get code 0.
template <class T>
__global__ void __launch_bounds__(256) mx_quantize_kernel(const T* __restrict__ x, int rows, int K,
                                                          uint8_t* __restrict__ packed,
                                                          uint8_t* __restrict__ sf) {
  const int groups = K / 32;
  const int groups_pad = (groups + 3) / 4 * 4;
  const int64_t rows_pad = (int64_t(rows) + 127) / 128 * 128;
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (idx >= rows_pad * groups_pad) return;
  const int64_t r = idx / groups_pad;
  const int64_t kg = idx - r * groups_pad;
  uint32_t code = 0;
  if (r < rows && kg < groups) {
    float v[32];
    float lo16[16], hi16[16];
    load16(x + r * K + kg * 32, lo16);
    load16(x + r * K + kg * 32 + 16, hi16);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = lo16[i];
      v[16 + i] = hi16[i];
    }
    float amax_b = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax_b = fmaxf(amax_b, fabsf(v[i]));
    const int ebits = static_cast<int>((__float_as_uint(amax_b) >> 23) & 0xFFu);
    int e = ebits == 0 ? -127 : ebits - 129;
    e = max(-127, min(127, e));
    code = static_cast<uint32_t>(e + 127);
    const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      w[q] = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) w[q] |= e2m1_rne(v[8 * q + i] * inv) << (4 * i);
    }
    *reinterpret_cast<uint4*>(packed + (r * K + kg * 32) / 2) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  sf[blackhole::sf_offset_vs(r, kg, K, 32)] = static_cast<uint8_t>(code);
}

// Two floats to two E4M3 bytes (round to nearest even, finite values past 448 saturate):
// lo in the low byte.
__device__ __forceinline__ uint32_t e4m3x2_satfinite(float lo, float hi) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(hi), "f"(lo));
  return d;
}

// MXFP8 (OCP MX v1.0, E4M3 elements): as mx_quantize_kernel with the E4M3 element exponent
// 8, e = floor(log2(amax_b)) - 8, and 32 bytes of E4M3 codes per group.
template <class T>
__global__ void __launch_bounds__(256) mx8_quantize_kernel(const T* __restrict__ x, int rows,
                                                           int K, uint8_t* __restrict__ q,
                                                           uint8_t* __restrict__ sf) {
  const int groups = K / 32;
  const int groups_pad = (groups + 3) / 4 * 4;
  const int64_t rows_pad = (int64_t(rows) + 127) / 128 * 128;
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (idx >= rows_pad * groups_pad) return;
  const int64_t r = idx / groups_pad;
  const int64_t kg = idx - r * groups_pad;
  uint32_t code = 0;
  if (r < rows && kg < groups) {
    float v[32];
    float lo16[16], hi16[16];
    load16(x + r * K + kg * 32, lo16);
    load16(x + r * K + kg * 32 + 16, hi16);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = lo16[i];
      v[16 + i] = hi16[i];
    }
    float amax_b = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax_b = fmaxf(amax_b, fabsf(v[i]));
    const int ebits = static_cast<int>((__float_as_uint(amax_b) >> 23) & 0xFFu);
    int e = ebits == 0 ? -127 : ebits - 135;
    e = max(-127, min(127, e));
    code = static_cast<uint32_t>(e + 127);
    const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w[i] = e4m3x2_satfinite(v[4 * i] * inv, v[4 * i + 1] * inv) |
             (e4m3x2_satfinite(v[4 * i + 2] * inv, v[4 * i + 3] * inv) << 16);
    uint4* dst = reinterpret_cast<uint4*>(q + r * K + kg * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
  sf[blackhole::sf_offset_vs(r, kg, K, 32)] = static_cast<uint8_t>(code);
}

}  // namespace quant_detail

// X: rows x K (FP32 if x_is_bf16 == 0, else BF16), K % 16 == 0, 16-byte aligned.
// packed: rows*K/2 bytes.  sf: sf_storage_bytes(rows, K) bytes (every padding byte written 0).
// scales: device float[2]; on completion scales[0] = amax, scales[1] = global scale g.
inline cudaError_t nvfp4_quantize(const void* X, int x_is_bf16, int rows, int K, void* packed,
                                  void* sf, float* scales, cudaStream_t stream = nullptr) {
  if (rows < 1 || K < 16 || K % 16 != 0 || !X || !packed || !sf || !scales)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(X) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 7u) ||
      (reinterpret_cast<uintptr_t>(scales) & 7u))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(scales, 0, 2 * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n16 = int64_t(rows) * K / 16;
  const int amax_grid = static_cast<int>(std::min<int64_t>((n16 + 255) / 256, int64_t(sms) * 8));
  const int64_t work = (int64_t(rows) + 127) / 128 * 128 * ((K / 16 + 3) / 4 * 4);
  const int64_t qgrid = (work + 255) / 256;
  if (qgrid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  if (x_is_bf16) {
    auto xp = static_cast<const __nv_bfloat16*>(X);
    quant_detail::amax_kernel<<<amax_grid, 256, 0, stream>>>(xp, n16, scales);
    quant_detail::quantize_kernel<<<static_cast<int>(qgrid), 256, 0, stream>>>(
        xp, rows, K, static_cast<uint8_t*>(packed), static_cast<uint8_t*>(sf), scales);
  } else {
    auto xp = static_cast<const float*>(X);
    quant_detail::amax_kernel<<<amax_grid, 256, 0, stream>>>(xp, n16, scales);
    quant_detail::quantize_kernel<<<static_cast<int>(qgrid), 256, 0, stream>>>(
        xp, rows, K, static_cast<uint8_t*>(packed), static_cast<uint8_t*>(sf), scales);
  }
  return cudaGetLastError();
}

// MXFP4 quantiser: X rows x K (FP32 if x_is_bf16 == 0, else BF16), K % 32 == 0, 16-byte
// aligned.  packed: rows*K/2 bytes (16-byte aligned).  sf: sf_storage_bytes_vs(rows, K, 32)
// bytes, every padding byte written 0.  No global scale: alpha of an MXFP4 GEMM is 1 (or the
// caller's own).
inline cudaError_t mxfp4_quantize(const void* X, int x_is_bf16, int rows, int K, void* packed,
                                  void* sf, cudaStream_t stream = nullptr) {
  if (rows < 1 || K < 32 || K % 32 != 0 || !X || !packed || !sf) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(X) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 15u))
    return cudaErrorInvalidValue;
  const int64_t work = (int64_t(rows) + 127) / 128 * 128 * ((K / 32 + 3) / 4 * 4);
  const int64_t grid = (work + 255) / 256;
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  if (x_is_bf16)
    quant_detail::mx_quantize_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(X), rows, K, static_cast<uint8_t*>(packed),
        static_cast<uint8_t*>(sf));
  else
    quant_detail::mx_quantize_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
        static_cast<const float*>(X), rows, K, static_cast<uint8_t*>(packed),
        static_cast<uint8_t*>(sf));
  return cudaGetLastError();
}

// MXFP8 quantiser: X rows x K (FP32 if x_is_bf16 == 0, else BF16), K % 32 == 0, 16-byte
// aligned.  q: rows*K bytes of E4M3 (16-byte aligned).  sf: sf_storage_bytes_vs(rows, K, 32)
// bytes, every padding byte written 0.
inline cudaError_t mxfp8_quantize(const void* X, int x_is_bf16, int rows, int K, void* q,
                                  void* sf, cudaStream_t stream = nullptr) {
  if (rows < 1 || K < 32 || K % 32 != 0 || !X || !q || !sf) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(X) & 15u) || (reinterpret_cast<uintptr_t>(q) & 15u))
    return cudaErrorInvalidValue;
  const int64_t work = (int64_t(rows) + 127) / 128 * 128 * ((K / 32 + 3) / 4 * 4);
  const int64_t grid = (work + 255) / 256;
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  if (x_is_bf16)
    quant_detail::mx8_quantize_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(X), rows, K, static_cast<uint8_t*>(q),
        static_cast<uint8_t*>(sf));
  else
    quant_detail::mx8_quantize_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(
        static_cast<const float*>(X), rows, K, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf));
  return cudaGetLastError();
}

#endif  // __CUDACC__

}  // namespace blackhole::sm100
