// make_golden.cpp -- writes the golden vectors that pin the CPU oracle (oracle/).
//
// Built and run by tests/golden/make_golden.sh in a container that holds the reference tree
// (Jiaao-Bai/blackhole) and CUTLASS 4.5.0 headers.  Everything written here comes from the
// reference's own code paths:
//   * conversions: cutlass::float_e2m1_t / float_ue4m3_t / bfloat16_t host constructors, the
//     converters the reference example calls (example/nvfp4_bf16_gemm.cu:61-71, :168);
//   * scale-factor offsets: blackhole::sm120::make_layout_SFA / make_layout_SFB
//     (include/blackhole/sm120/nvfp4_gemm.hpp:293-298), evaluated on the host;
//   * small GEMMs: inputs drawn the way the example draws them (mt19937(1234), FP4 levels
//     {-2,-1,-0.5,0,0.5,1,2}, scale levels {0.5,1,1,2}, example:98-133) and the example's
//     sequential FP32 host loop (example:161-168) evaluated at every output element.
//
// Output: little-endian raw arrays in the current directory plus manifest.json.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include <blackhole/sm120/nvfp4_gemm.hpp>

namespace {

std::string g_manifest = "{\n";
bool g_first = true;

template <class T>
void dump(const char* name, const std::vector<T>& v, const char* dtype) {
  FILE* f = std::fopen(name, "wb");
  std::fwrite(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
  char buf[256];
  std::snprintf(buf, sizeof buf, "%s  \"%s\": {\"dtype\": \"%s\", \"count\": %zu}",
                g_first ? "" : ",\n", name, dtype, v.size());
  g_first = false;
  g_manifest += buf;
}

float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

uint32_t lcg(uint64_t& s) {
  s = s * 6364136223846793005ull + 1442695040888963407ull;
  return uint32_t(s >> 32);
}

void conversions() {
  // (1) every bf16 bit pattern widened to f32: all exponents, 7-bit mantissas, +-0, inf, NaN.
  std::vector<float> in;
  for (uint32_t b = 0; b < 65536; ++b) in.push_back(u2f(b << 16));
  // (2) f32 patterns with full 23-bit mantissas near the e2m1 / ue4m3 ranges.
  uint64_t s = 0x1234;
  for (int i = 0; i < 16384; ++i) {
    uint32_t r = lcg(s);
    int e = 127 - 12 + int(r % 23);                 // 2^-12 .. 2^10
    uint32_t mant = lcg(s) & 0x7FFFFF;
    uint32_t sign = (r >> 31) << 31;
    in.push_back(u2f(sign | (uint32_t(e) << 23) | mant));
  }
  // (3) exact midpoints and their neighbours for both formats.
  const float ties[] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f, 6.0f, 7.0f};
  for (float t : ties) {
    in.push_back(t); in.push_back(-t);
    in.push_back(std::nextafter(t, 0.f)); in.push_back(std::nextafter(t, 100.f));
  }
  for (int e = -10; e <= 9; ++e)
    for (int m = 0; m < 16; ++m) {
      float t = std::ldexp(1.0f + m / 16.0f, e);     // ue4m3 midpoints when m is odd
      in.push_back(t); in.push_back(std::nextafter(t, 0.f)); in.push_back(std::nextafter(t, 1e9f));
    }
  std::vector<uint8_t> e2m1(in.size()), ue4m3(in.size());
  for (size_t i = 0; i < in.size(); ++i) {
    e2m1[i] = cutlass::float_e2m1_t(in[i]).storage & 0xF;
    ue4m3[i] = cutlass::float_ue4m3_t(in[i]).storage;
  }
  dump("conv_in.f32", in, "float32");
  dump("conv_e2m1.u8", e2m1, "uint8");
  dump("conv_ue4m3.u8", ue4m3, "uint8");

  // bf16 rounding over arbitrary f32 patterns (all exponents) plus exact ties.
  std::vector<float> bin;
  s = 0xbf16;
  for (int i = 0; i < 65536; ++i) bin.push_back(u2f(lcg(s)));
  for (int i = 0; i < 4096; ++i) {
    uint32_t hi = lcg(s) & 0xFFFF0000u;
    bin.push_back(u2f(hi | 0x8000u));                // exact tie
    bin.push_back(u2f(hi | 0x7FFFu));
    bin.push_back(u2f(hi | 0x8001u));
  }
  std::vector<uint16_t> bout(bin.size());
  for (size_t i = 0; i < bin.size(); ++i) bout[i] = cutlass::bfloat16_t(bin[i]).storage;
  dump("bf16_in.f32", bin, "float32");
  dump("bf16_out.u16", bout, "uint16");

  // decode tables
  std::vector<float> dec_e2m1(16), dec_ue4m3(256);
  for (int c = 0; c < 16; ++c) dec_e2m1[c] = float(cutlass::float_e2m1_t::bitcast(uint8_t(c)));
  for (int c = 0; c < 256; ++c) dec_ue4m3[c] = float(cutlass::float_ue4m3_t::bitcast(uint8_t(c)));
  dump("dec_e2m1.f32", dec_e2m1, "float32");
  dump("dec_ue4m3.f32", dec_ue4m3, "float32");
}

void sf_layouts() {
  struct S { int mn, k; };
  const S shapes[] = {{128, 256}, {256, 512}, {384, 1024}, {16, 512}, {1, 256},
                      {200, 768}, {130, 320}, {64, 8192}};
  for (const S& sh : shapes) {
    auto la = blackhole::sm120::make_layout_SFA(sh.mn, sh.k);
    auto lb = blackhole::sm120::make_layout_SFB(sh.mn, sh.k);
    const int kg = sh.k / 16;
    std::vector<int64_t> off;
    off.push_back(int64_t(cute::cosize(la)));
    off.push_back(int64_t(cute::cosize(lb)));
    for (int m = 0; m < sh.mn; ++m)
      for (int g = 0; g < kg; ++g) {
        int64_t a = la(cute::make_coord(m, g * 16));
        int64_t b = lb(cute::make_coord(m, g * 16));
        if (a != b) { std::fprintf(stderr, "SFA/SFB layouts differ\n"); std::exit(1); }
        off.push_back(a);
      }
    char name[64];
    std::snprintf(name, sizeof name, "sf_%dx%d.i64", sh.mn, sh.k);
    dump(name, off, "int64");
  }
  // a large decode-shaped layout: cosize only (the offsets follow the same rule)
  std::vector<int64_t> big = {int64_t(cute::cosize(blackhole::sm120::make_layout_SFA(16, 8192))),
                              int64_t(cute::cosize(blackhole::sm120::make_layout_SFB(28672, 8192)))};
  dump("sf_cosize_decode.i64", big, "int64");
}

// Inputs drawn in the example's order, then its host loop at every (m, n).
void example_gemm(int M, int N, int K) {
  const int Kg = K / 16;
  auto la = blackhole::sm120::make_layout_SFA(M, K);
  auto lb = blackhole::sm120::make_layout_SFB(N, K);
  std::vector<uint8_t> A(size_t(M) * K / 2), B(size_t(N) * K / 2);
  std::vector<uint8_t> SFA(cute::cosize(la)), SFB(cute::cosize(lb));
  std::vector<float> av(size_t(M) * K), bv(size_t(N) * K), sa(size_t(M) * Kg), sb(size_t(N) * Kg);
  std::mt19937 rng(1234);
  std::uniform_int_distribution<int> pick(0, 6), pick_sf(0, 3);
  const float lv[7] = {-2.f, -1.f, -0.5f, 0.f, 0.5f, 1.f, 2.f};
  const float sl[4] = {0.5f, 1.f, 1.f, 2.f};
  auto fill = [&](int rows, auto& layout, std::vector<uint8_t>& P, std::vector<uint8_t>& SF,
                  std::vector<float>& vals, std::vector<float>& sfv) {
    for (int r = 0; r < rows; ++r) {
      for (int g = 0; g < Kg; ++g) {
        cutlass::float_ue4m3_t q(sl[pick_sf(rng)]);
        SF[layout(cute::make_coord(r, g * 16))] = q.storage;
        sfv[size_t(r) * Kg + g] = float(q);
      }
      for (int k = 0; k < K; ++k) {
        cutlass::float_e2m1_t q(lv[pick(rng)]);
        uint8_t code = q.storage & 0xF;
        vals[size_t(r) * K + k] = float(q);
        size_t byte = (size_t(r) * K + k) / 2;
        P[byte] = (k & 1) ? uint8_t((P[byte] & 0x0F) | (code << 4)) : uint8_t((P[byte] & 0xF0) | code);
      }
    }
  };
  fill(M, la, A, SFA, av, sa);
  fill(N, lb, B, SFB, bv, sb);
  std::vector<uint16_t> D(size_t(M) * N);
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      float acc = 0.f;
      for (int k = 0; k < K; ++k) {
        float a = av[size_t(m) * K + k] * sa[size_t(m) * Kg + k / 16];
        float b = bv[size_t(n) * K + k] * sb[size_t(n) * Kg + k / 16];
        acc += a * b;
      }
      D[size_t(m) * N + n] = cutlass::bfloat16_t(acc).storage;
    }
  char name[96];
  std::snprintf(name, sizeof name, "gemm_%dx%dx%d_A.u8", M, N, K);   dump(name, A, "uint8");
  std::snprintf(name, sizeof name, "gemm_%dx%dx%d_SFA.u8", M, N, K); dump(name, SFA, "uint8");
  std::snprintf(name, sizeof name, "gemm_%dx%dx%d_B.u8", M, N, K);   dump(name, B, "uint8");
  std::snprintf(name, sizeof name, "gemm_%dx%dx%d_SFB.u8", M, N, K); dump(name, SFB, "uint8");
  std::snprintf(name, sizeof name, "gemm_%dx%dx%d_D.u16", M, N, K);  dump(name, D, "uint16");
}

}  // namespace

int main() {
  conversions();
  sf_layouts();
  example_gemm(128, 128, 256);
  example_gemm(256, 384, 512);
  g_manifest += "\n}\n";
  FILE* f = std::fopen("manifest.json", "w");
  std::fputs(g_manifest.c_str(), f);
  std::fclose(f);
  return 0;
}
