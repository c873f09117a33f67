#pragma once

// Element / scale-factor formats the sm_100a block-scaled GEMM serves.  Both use E2M1
// elements (two per byte, K-contiguous) and the 128x4 blocked scale-factor layout; they
// differ in the scale-factor type and in how many elements one scale factor covers:
//
//   * NVFP4 (the reference's format): one UE4M3 scale per 16 elements, plus the global
//     scale folded into alpha;
//   * MXFP4 (OCP Microscaling v1.0): one UE8M0 scale (a power of two) per 32 elements.
//
// Both run on tcgen05.mma kind::mxf4nvf4, with 16- or 32-element scale blocks.

#include <cstdint>

namespace blackhole::sm100 {

struct Nvfp4Format {
  static constexpr int SfVec = 16;            // elements per scale factor
  static constexpr uint32_t ScaleType = 0;    // instruction-descriptor scale format: UE4M3
};

struct Mxfp4Format {
  static constexpr int SfVec = 32;
  static constexpr uint32_t ScaleType = 1;    // UE8M0
};

}  // namespace blackhole::sm100
