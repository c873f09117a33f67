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
// a grid-stride amax reduction, then the quantiser proper with two lanes per 16-element
// block (a warp reads 1 KB of contiguous FP32 and stores 128 contiguous bytes of codes).
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

// Four E2M1 codes of q[0..3] (round to nearest even, finite values past 6 saturate), q[0] in
// the lowest nibble.  cvt...e2m1x2 puts its first source in the upper nibble.
__device__ __forceinline__ uint32_t e2m1x4_cvt(float q0, float q1, float q2, float q3) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "mov.b32 %0, {b0, b1, b0, b1};\n\t}"
      : "=r"(out)
      : "f"(q0), "f"(q1), "f"(q2), "f"(q3));
  return out & 0xFFFFu;
}
// UE4M3 code of v >= 0 (round to nearest even, saturating at 448): the E4M3 conversion of a
// non-negative value, whose sign bit is then 0.
__device__ __forceinline__ uint32_t ue4m3_cvt(float v) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(0.0f), "f"(v));
  return d & 0xFFu;
}

// The recipe's roundings are of exact IEEE quotients: s = UE4M3(fl(fl(amax_b / 6) / g)) and
// q = E2M1(fl(x / fl(s * g))).  Both conversions are monotone with rounding thresholds of few
// significant bits (E2M1: the midpoints 0.25, 0.75, ..., 5, three bits; UE4M3: midpoints of
// values with four, five bits), so they are computed from a cheap estimate y of the quotient
// (products with reciprocals; within 6 units in the last place of the quotient) unless y lies
// within 16 (E2M1) or 32 (UE4M3) representable floats of a value with that few significant
// bits -- its low 21 (19) fraction bits, offset by the window, wrap into the window.  Then the
// exact division is made.  A quotient that far from every threshold rounds like its estimate,
// so the results are bit-identical to the plain recipe; the exact path runs for a few
// elements in a million.
__device__ __forceinline__ bool near_e2m1_threshold(float y) {
  return ((__float_as_uint(y) + 16u) & 0x1FFFFFu) < 33u;
}
__device__ __forceinline__ bool near_ue4m3_threshold(float y) {
  return ((__float_as_uint(y) + 32u) & 0x7FFFFu) < 65u;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Eight consecutive elements of a lane (32 bytes of FP32 in two 16-byte loads that the same
// warp's next load finds in L1, or one 16-byte load of BF16).
template <class T> struct Vec8In;
template <> struct Vec8In<float> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};
template <> struct Vec8In<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};

// Work item: 256 consecutive elements of one row (a segment), one warp, 8 elements per lane,
// so one 16-element block is 2 neighbouring lanes.  Each warp takes a contiguous range of
// items (row-major: segments of a row, then the next row), so it steps through rows without
// dividing.  Items run over the layout's padded rows (a multiple of 128); items of padding
// rows and the groups past K of a row's last segment write zero scale factors.  Every
// scale-factor write is one 4-byte word (4 groups of one row) by lanes 0, 8, 16, 24; codes are
// 32-bit stores, 128 contiguous bytes per warp.
template <class T, int kItemsPerWarp>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ x, int rows, int K,
                                                       uint8_t* __restrict__ packed,
                                                       uint8_t* __restrict__ sf,
                                                       float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int segs = (K + 255) / 256;
  const int rows_pad = (rows + 127) / 128 * 128;
  const int words_per_row = (K / 16 + 3) / 4;          // 4-group words (the padded groups)
  const int items = rows_pad * segs;                   // < 2^31: checked by the launcher
  const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  int it = warp * kItemsPerWarp;
  const int it_end = min(items, it + kItemsPerWarp);
  const float amax = scales[0];
  const float g = amax / 2688.0f;                       // amax / (448 * 6)
  if (blockIdx.x == 0 && threadIdx.x == 0) scales[1] = g;
  // (amax_b / 6) / g ~ amax_b * c: fl(1/6), fl(1/g) and their product, three roundings
  const float c = __frcp_rn(6.0f) * __frcp_rn(g);
  if (it >= it_end) return;
  int r = it / segs;
  int seg = it - r * segs;
  constexpr int U = 2;                                  // items whose loads are in flight together
  for (; it < it_end; it += U) {
    float v[U][8];
    int ru[U], k0[U];
    bool live[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      ru[u] = r;
      k0[u] = seg * 256 + lane * 8;
      live[u] = it + u < it_end && r < rows && k0[u] < K;
      if (live[u]) {
        Vec8In<T>::load(x + int64_t(r) * K + k0[u], v[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[u][i] = 0.0f;
      }
      if (++seg == segs) {
        seg = 0;
        ++r;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (it + u >= it_end) break;                      // warp-uniform
      float m = fabsf(v[u][0]);
#pragma unroll
      for (int i = 1; i < 8; ++i) m = fmaxf(m, fabsf(v[u][i]));
      m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));   // the block's amax on its 2 lanes
      uint32_t s_code = 0, codes = 0;
      if (live[u] && g > 0.0f && m > 0.0f) {
        const float ys = m * c;
        s_code = near_ue4m3_threshold(ys) ? ue4m3_cvt((m / 6.0f) / g) : ue4m3_cvt(ys);
        const float s_val = ue4m3_value(s_code);
        if (s_val != 0.0f) {
          const float scale = s_val * g;
          const float rs = rcp_approx(scale);       // subnormal scale: inf, every y "near"
          float y[8];
          bool near = false;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            y[i] = v[u][i] * rs;
            near |= near_e2m1_threshold(y[i]);
          }
          if (near) {
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = v[u][i] / scale;
          }
          codes = e2m1x4_cvt(y[0], y[1], y[2], y[3]) | (e2m1x4_cvt(y[4], y[5], y[6], y[7]) << 16);
        }
      }
      if (live[u]) *reinterpret_cast<uint32_t*>(packed + (int64_t(ru[u]) * K + k0[u]) / 2) = codes;
      // the 16 groups of the segment as four words: lanes 0, 2, 4, 6 -> word 0, lanes 8..14 ->
      // word 1, ...; word w is assembled on lanes 8w..8w+3 and stored by lane 8w
      const uint32_t cw = __shfl_sync(0xFFFFFFFFu, s_code, (lane & 24) + 2 * (lane & 3))
                          << (8 * (lane & 3));
      uint32_t word = cw | __shfl_xor_sync(0xFFFFFFFFu, cw, 1);
      word |= __shfl_xor_sync(0xFFFFFFFFu, word, 2);
      const int w = (k0[u] - lane * 8) / 64 + (lane >> 3);   // this lane's word of the row
      if ((lane & 7) == 0 && w < words_per_row && ru[u] < rows_pad)
        *reinterpret_cast<uint32_t*>(sf + blackhole::sf_offset(ru[u], 4 * w, K)) = word;
    }
  }
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
  // quantiser: 8 warps per CTA, each warp a contiguous range of kItems segments of 256
  // elements (one pass over the tensor, ~10 warps per SM for the configs' shapes and more)
  constexpr int kItems = 16;
  const int64_t items = (int64_t(rows) + 127) / 128 * 128 * ((K + 255) / 256);
  if (items >= (int64_t(1) << 31) - (int64_t(1) << 20)) return cudaErrorInvalidValue;
  const int qgrid = static_cast<int>(std::max<int64_t>(1, (items + 8 * kItems - 1) / (8 * kItems)));
  if (x_is_bf16) {
    auto xp = static_cast<const __nv_bfloat16*>(X);
    quant_detail::amax_kernel<<<amax_grid, 256, 0, stream>>>(xp, n16, scales);
    quant_detail::quantize_kernel<__nv_bfloat16, kItems><<<qgrid, 256, 0, stream>>>(
        xp, rows, K, static_cast<uint8_t*>(packed), static_cast<uint8_t*>(sf), scales);
  } else {
    auto xp = static_cast<const float*>(X);
    quant_detail::amax_kernel<<<amax_grid, 256, 0, stream>>>(xp, n16, scales);
    quant_detail::quantize_kernel<float, kItems><<<qgrid, 256, 0, stream>>>(
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
