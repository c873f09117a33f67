// Golden vectors for the MXFP4 sibling format, produced by CUTLASS 4.5.0's own host code
// (the reference has no MX path; these pin the oracle's MX parts the way make_golden.cpp pins
// the NVFP4 parts):
//   * mx_dec_ue8m0.f32: cutlass::float_ue8m0_t decoded for all 256 codes;
//   * mx_sf_<mn>x<k>.i64: cosize of the SFA and SFB layouts, then the byte offset of every
//     (row, 32-element K group) of cutlass::detail::Sm1xxBlockScaledConfig<32>'s layouts;
//   * mx_dec_e4m3.f32: cutlass::float_e4m3_t decoded for all 256 codes;
//   * mx_e4m3_in.f32 / mx_e4m3_out.u8: cutlass::float_e4m3_t(float) (host conversion) of
//     every bf16 bit pattern, 16384 seeded random floats and every midpoint between
//     adjacent E4M3 magnitudes (the MXFP8 element encoding).
// Build and run with make_golden_mx.sh; writes next to itself, with manifest_mx.json.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <cute/tensor.hpp>
#include <cutlass/float8.h>
#include <cutlass/detail/sm100_blockscaled_layout.hpp>

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

using MxConfig = cutlass::detail::Sm1xxBlockScaledConfig<32>;

void decode_table() {
  std::vector<float> dec(256);
  for (int c = 0; c < 256; ++c) dec[c] = float(cutlass::float_ue8m0_t::bitcast(uint8_t(c)));
  dump("mx_dec_ue8m0.f32", dec, "float32");
}

void e4m3() {
  std::vector<float> dec(256);
  for (int c = 0; c < 256; ++c) dec[c] = float(cutlass::float_e4m3_t::bitcast(uint8_t(c)));
  dump("mx_dec_e4m3.f32", dec, "float32");
  std::vector<float> in;
  for (uint32_t h = 0; h < 65536; ++h) {
    const uint32_t u = h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    in.push_back(f);
  }
  uint64_t z = 0x9E3779B97F4A7C15ull;
  for (int i = 0; i < 16384; ++i) {   // splitmix64 bits as float magnitudes up to ~2^10
    z += 0x9E3779B97F4A7C15ull;
    uint64_t t = z;
    t = (t ^ (t >> 30)) * 0xBF58476D1CE4E5B9ull;
    t = (t ^ (t >> 27)) * 0x94D049BB133111EBull;
    t ^= t >> 31;
    const uint32_t u = (uint32_t(t) & 0x807FFFFFu) | (uint32_t(((t >> 32) % 30) + 104) << 23);
    float f;
    std::memcpy(&f, &u, 4);
    in.push_back(f);
  }
  for (int c = 0; c < 0x7E; ++c) {    // midpoints between adjacent magnitudes, both signs
    const float lo = float(cutlass::float_e4m3_t::bitcast(uint8_t(c)));
    const float hi = float(cutlass::float_e4m3_t::bitcast(uint8_t(c + 1)));
    in.push_back(0.5f * (lo + hi));
    in.push_back(-0.5f * (lo + hi));
  }
  std::vector<uint8_t> out;
  for (float f : in) out.push_back(cutlass::float_e4m3_t(f).storage);
  dump("mx_e4m3_in.f32", in, "float32");
  dump("mx_e4m3_out.u8", out, "uint8");
}

void layouts() {
  struct S { int mn, k; };
  const S shapes[] = {{128, 256}, {256, 512}, {200, 768}, {16, 1024}, {130, 320}, {1, 128}};
  for (const S& sh : shapes) {
    auto la = MxConfig::tile_atom_to_shape_SFA(cute::make_shape(sh.mn, 0, sh.k));
    auto lb = MxConfig::tile_atom_to_shape_SFB(cute::make_shape(0, sh.mn, sh.k));
    std::vector<int64_t> off;
    off.push_back(int64_t(cute::cosize(la)));
    off.push_back(int64_t(cute::cosize(lb)));
    for (int m = 0; m < sh.mn; ++m)
      for (int g = 0; g < sh.k / 32; ++g) {
        const int64_t a = la(cute::make_coord(m, g * 32));
        const int64_t b = lb(cute::make_coord(m, g * 32));
        if (a != b) { std::fprintf(stderr, "SFA / SFB layouts differ\n"); std::exit(1); }
        off.push_back(a);
      }
    char name[64];
    std::snprintf(name, sizeof name, "mx_sf_%dx%d.i64", sh.mn, sh.k);
    dump(name, off, "int64");
  }
}

}  // namespace

int main() {
  decode_table();
  layouts();
  e4m3();
  g_manifest += "\n}\n";
  FILE* f = std::fopen("manifest_mx.json", "w");
  std::fputs(g_manifest.c_str(), f);
  std::fclose(f);
  return 0;
}
