#pragma once

// Architecture traits for the Blackwell targets.
//
// Same surface as the reference's include/blackhole/common/arch.hpp:15-42 (Arch enum,
// arch_traits<Arch>::sm / has_tcgen05, BLACKHOLE_ARCH_SM100/SM120 macros from
// __CUDA_ARCH__), extended with the sm_100 resource figures the B200 kernels size
// themselves against.  It has no CuTe dependency.

namespace blackhole {

enum class Arch {
  kSm100,
  kSm120,
};

template <Arch A>
struct arch_traits;

template <>
struct arch_traits<Arch::kSm100> {
  static constexpr int sm           = 100;
  static constexpr bool has_tcgen05 = true;
  // B200: 148 SMs on two dies.  The launcher queries the live count; this is the default.
  static constexpr int num_sms               = 148;
  static constexpr int max_smem_per_cta      = 232448;  // 227 KB opt-in dynamic smem
  static constexpr int tmem_columns          = 512;     // 32-bit columns per SM
  static constexpr int tmem_lanes            = 128;
  static constexpr int max_cluster_portable  = 8;
};

template <>
struct arch_traits<Arch::kSm120> {
  static constexpr int sm           = 120;
  static constexpr bool has_tcgen05 = false;
};

// Compile-time current target convenience macros.
#if defined(__CUDA_ARCH__)
#  if (__CUDA_ARCH__ >= 1000) && (__CUDA_ARCH__ < 1200)
#    define BLACKHOLE_ARCH_SM100 1
#  elif (__CUDA_ARCH__ >= 1200) && (__CUDA_ARCH__ < 1300)
#    define BLACKHOLE_ARCH_SM120 1
#  endif
#endif

}  // namespace blackhole
