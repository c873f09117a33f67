// ref_shim.cpp -- exposes the reference's own host code paths through a C ABI so the tests
// can check the oracle restatement against them point by point.  TEST INFRASTRUCTURE ONLY.
//
// Compiled by `make -C oracle ref` from the reference tree where it lies (read-only) plus
// CUTLASS 4.5.0 headers; the result goes to oracle/_ref/libref_shim.so.  Nothing is copied.
//   ref_sf_offset / ref_sf_cosize : blackhole::sm120::make_layout_SFA/SFB
//                                   (include/blackhole/sm120/nvfp4_gemm.hpp:293-298)
//   ref_e2m1 / ref_ue4m3 / ref_bf16: the CUTLASS converters the example calls
//                                   (example/nvfp4_bf16_gemm.cu:61-71, :168)
#include <cstdint>

#include <blackhole/sm120/nvfp4_gemm.hpp>

extern "C" {

int64_t ref_sf_offset(int64_t mn, int64_t kg, int64_t MN, int64_t K, int is_b) {
  if (is_b) return blackhole::sm120::make_layout_SFB(int(MN), int(K))(cute::make_coord(int(mn), int(kg * 16)));
  return blackhole::sm120::make_layout_SFA(int(MN), int(K))(cute::make_coord(int(mn), int(kg * 16)));
}

int64_t ref_sf_cosize(int64_t MN, int64_t K, int is_b) {
  if (is_b) return cute::cosize(blackhole::sm120::make_layout_SFB(int(MN), int(K)));
  return cute::cosize(blackhole::sm120::make_layout_SFA(int(MN), int(K)));
}

uint8_t ref_e2m1(float x) { return cutlass::float_e2m1_t(x).storage & 0xF; }
uint8_t ref_ue4m3(float x) { return cutlass::float_ue4m3_t(x).storage; }
uint16_t ref_bf16(float x) { return cutlass::bfloat16_t(x).storage; }
float ref_ue4m3_decode(uint8_t c) { return float(cutlass::float_ue4m3_t::bitcast(c)); }

}  // extern "C"
