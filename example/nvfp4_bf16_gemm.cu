// =====================================================================================
// blackhole sm100 NVFP4 x NVFP4 -> BF16 GEMM: runnable example, self-check and timing.
// -------------------------------------------------------------------------------------
// The B200 (sm_100a) counterpart of the reference's example/nvfp4_bf16_gemm.cu: the same
// flow -- NVFP4 inputs drawn from a few exactly representable levels, the operator called
// with the reference's nine arguments, a sampled check against the host loop, and a timed
// loop reporting TFLOP/s -- written against blackhole::sm100.  A caller of the reference
// changes only the namespace (sm120 -> sm100) and the header path.
//
//   ./nvfp4_bf16_gemm_sm100 [M N K] [--iters I] [--samples S]     (default 4096 4096 4096)
//
// The file builds two ways (CMakeLists.txt builds both):
//   * with nvcc (-gencode arch=compute_100a,code=sm_100a): the header-only operator, its
//     kernels compiled into this program -- the reference's own way of using its header;
//   * with a host C++ compiler (example/nvfp4_bf16_gemm_capi.cpp includes this file): the
//     same header then forwards the call to the C ABI of libblackhole_sm100.so.
// Exit code 0 when every sampled element matches (rel <= 0.05, the reference's check; with
// these inputs every partial sum is exact in FP32, so the GPU result must also equal the
// host loop's BF16 bit for bit, which is reported and required).
// =====================================================================================
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include <cuda_runtime_api.h>

#include <blackhole/common/sf_layout.hpp>
#include <blackhole/sm100/nvfp4_gemm.hpp>

using namespace blackhole::sm100;

namespace {

constexpr int kSfVec = 16;   // one UE4M3 scale per 16 elements along K

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "CUDA error in %s: %s\n", what, cudaGetErrorString(e));
    std::exit(2);
  }
}

// Value of each 4-bit E2M1 code (sign in bit 3) and of each 8-bit UE4M3 code (bit 7 unused).
float e2m1_value(uint8_t code) {
  static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  return (code & 8) ? -mag[code & 7] : mag[code & 7];
}
float ue4m3_value(uint8_t code) {
  const int e = (code >> 3) & 15, m = code & 7;
  if (e == 0) return std::ldexp(float(m), -9);              // subnormal: m/8 * 2^-6
  return std::ldexp(1.f + m / 8.f, e - 7);
}
// Code of an exactly representable value (the levels below are), found by search.
uint8_t e2m1_code(float v) {
  for (uint8_t c = 0; c < 16; ++c)
    if (e2m1_value(c) == v) return c;
  std::fprintf(stderr, "%g is not an E2M1 value\n", v);
  std::exit(2);
}
uint8_t ue4m3_code(float v) {
  for (int c = 0; c < 127; ++c)
    if (ue4m3_value(uint8_t(c)) == v) return uint8_t(c);
  std::fprintf(stderr, "%g is not a UE4M3 value\n", v);
  std::exit(2);
}

uint16_t bf16_bits_rne(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0x7FFF;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
float bf16_value(uint16_t b) {
  const uint32_t u = uint32_t(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// One NVFP4 operand (rows x K): packed codes, scale factors in the 128x4 layout, and the
// decoded element and scale values the host loop uses.
struct Operand {
  std::vector<uint8_t> packed, sf;
  std::vector<float> val, scale;
};

Operand make_operand(int rows, int K, std::mt19937& rng) {
  static const float levels[7] = {-2.f, -1.f, -0.5f, 0.f, 0.5f, 1.f, 2.f};
  static const float scales[4] = {0.5f, 1.f, 1.f, 2.f};
  std::uniform_int_distribution<int> pick_level(0, 6), pick_scale(0, 3);
  const int groups = K / kSfVec;
  Operand o;
  o.packed.assign(size_t(rows) * K / 2, 0);
  o.sf.assign(size_t(blackhole::sf_storage_bytes(rows, K)), 0);
  o.val.resize(size_t(rows) * K);
  o.scale.resize(size_t(rows) * groups);
  for (int r = 0; r < rows; ++r) {
    for (int g = 0; g < groups; ++g) {
      const float s = scales[pick_scale(rng)];
      o.sf[size_t(blackhole::sf_offset(r, g, K))] = ue4m3_code(s);
      o.scale[size_t(r) * groups + g] = s;
    }
    for (int k = 0; k < K; ++k) {
      const float v = levels[pick_level(rng)];
      const uint8_t c = e2m1_code(v);
      uint8_t& byte = o.packed[(size_t(r) * K + k) / 2];
      byte = (k & 1) ? uint8_t((byte & 0x0F) | (c << 4)) : uint8_t((byte & 0xF0) | c);
      o.val[size_t(r) * K + k] = v;
    }
  }
  return o;
}

}  // namespace

int main(int argc, char** argv) {
  int M = 4096, N = 4096, K = 4096, iters = 50, samples = 256;
  int pos = 0;
  for (int i = 1; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--iters") && i + 1 < argc) {
      iters = std::atoi(argv[++i]);
    } else if (!std::strcmp(argv[i], "--samples") && i + 1 < argc) {
      samples = std::atoi(argv[++i]);
    } else if (pos < 3) {
      (pos == 0 ? M : pos == 1 ? N : K) = std::atoi(argv[i]);
      ++pos;
    }
  }
  std::printf("blackhole sm100 NVFP4 x NVFP4 -> BF16 GEMM   M=%d N=%d K=%d\n", M, N, K);
  // This operator takes any M >= 1, N % 8 == 0, K % 32 == 0; the example's inputs use whole
  // 16-element scale groups.
  if (M < 1 || N < 8 || N % 8 || K < 32 || K % 32) {
    std::printf("shape not supported: needs M >= 1, N %% 8 == 0, K %% 32 == 0\n");
    return 1;
  }

  std::mt19937 rng(1234);
  Operand a = make_operand(M, K, rng);
  Operand b = make_operand(N, K, rng);

  void *dA, *dB, *dSFA, *dSFB, *dD;
  check(cudaMalloc(&dA, a.packed.size()), "cudaMalloc A");
  check(cudaMalloc(&dB, b.packed.size()), "cudaMalloc B");
  check(cudaMalloc(&dSFA, a.sf.size()), "cudaMalloc SFA");
  check(cudaMalloc(&dSFB, b.sf.size()), "cudaMalloc SFB");
  check(cudaMalloc(&dD, size_t(M) * N * 2), "cudaMalloc D");
  check(cudaMemcpy(dA, a.packed.data(), a.packed.size(), cudaMemcpyHostToDevice), "copy A");
  check(cudaMemcpy(dB, b.packed.data(), b.packed.size(), cudaMemcpyHostToDevice), "copy B");
  check(cudaMemcpy(dSFA, a.sf.data(), a.sf.size(), cudaMemcpyHostToDevice), "copy SFA");
  check(cudaMemcpy(dSFB, b.sf.data(), b.sf.size(), cudaMemcpyHostToDevice), "copy SFB");
  check(cudaMemset(dD, 0xFF, size_t(M) * N * 2), "memset D");   // NaN: unwritten shows

  // The reference's nine-argument call; only the namespace differs.
  check(nvfp4_bf16_gemm(M, N, K, dA, dSFA, dB, dSFB, dD), "nvfp4_bf16_gemm");
  check(cudaDeviceSynchronize(), "first GEMM");
  std::vector<uint16_t> hD(size_t(M) * N);
  check(cudaMemcpy(hD.data(), dD, hD.size() * 2, cudaMemcpyDeviceToHost), "copy D");

  // Sampled check against the host loop: acc += (a*sfa)*(b*sfb) in k order, then BF16.
  std::mt19937 pick(7);
  std::uniform_int_distribution<int> row(0, M - 1), col(0, N - 1);
  const int groups = K / kSfVec;
  int bad = 0, exact = 0;
  double max_rel = 0.0;
  for (int s = 0; s < samples; ++s) {
    const int m = row(pick), n = col(pick);
    float acc = 0.f;
    for (int k = 0; k < K; ++k) {
      const float x = a.val[size_t(m) * K + k] * a.scale[size_t(m) * groups + k / kSfVec];
      const float y = b.val[size_t(n) * K + k] * b.scale[size_t(n) * groups + k / kSfVec];
      acc += x * y;
    }
    const uint16_t ref_bits = bf16_bits_rne(acc);
    const uint16_t got_bits = hD[size_t(m) * N + n];
    const float ref = bf16_value(ref_bits), got = bf16_value(got_bits);
    const double rel = std::fabs(double(got) - ref) / (std::fabs(double(ref)) + 1e-3);
    if (!(rel <= max_rel)) max_rel = std::isnan(rel) ? INFINITY : rel;
    exact += got_bits == ref_bits;
    if (!(rel <= 0.05)) {
      if (bad < 8) std::printf("  mismatch (%d,%d): got %.4f ref %.4f\n", m, n, got, ref);
      ++bad;
    }
  }
  const bool passed = bad == 0 && exact == samples;
  std::printf("Checked %d elements: max_rel=%.4f, mismatches=%d, bit-identical=%d -> %s\n",
              samples, max_rel, bad, exact, passed ? "PASSED" : "FAILED");

  // Timing: one warm-up call, then `iters` calls between two events.
  cudaEvent_t t0, t1;
  check(cudaEventCreate(&t0), "event");
  check(cudaEventCreate(&t1), "event");
  check(nvfp4_bf16_gemm(M, N, K, dA, dSFA, dB, dSFB, dD), "warm-up");
  check(cudaDeviceSynchronize(), "warm-up");
  check(cudaEventRecord(t0), "record");
  for (int i = 0; i < iters; ++i) check(nvfp4_bf16_gemm(M, N, K, dA, dSFA, dB, dSFB, dD), "GEMM");
  check(cudaEventRecord(t1), "record");
  check(cudaEventSynchronize(t1), "sync");
  float ms = 0.f;
  check(cudaEventElapsedTime(&ms, t0, t1), "elapsed");
  ms /= iters > 0 ? iters : 1;
  std::printf("Avg %.4f ms   %.1f TFLOP/s\n", ms, 2.0 * M * N * K / (ms * 1e-3) / 1e12);

  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dSFA);
  cudaFree(dSFB);
  cudaFree(dD);
  return passed ? 0 : 1;
}
