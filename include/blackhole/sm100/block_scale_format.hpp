#pragma once

// Element / scale-factor formats the sm_100a block-scaled GEMM serves.  All use the 128x4
// blocked scale-factor layout and K-contiguous operands; A is the M x K operand
// (activations), B the N x K operand (weights):
//
//   * NVFP4 (the reference's format): E2M1 x E2M1, one UE4M3 scale per 16 elements, plus
//     the global scale folded into alpha -- tcgen05.mma kind::mxf4nvf4, block16;
//   * MXFP4 (OCP Microscaling v1.0): E2M1 x E2M1, one UE8M0 scale (a power of two) per 32
//     elements -- kind::mxf4nvf4, block32;
//   * MXFP8 x MXFP4: E4M3 A (one byte per element) x E2M1 B, UE8M0 scales per 32 elements
//     on both -- kind::mxf8f6f4, where every element takes one byte in shared memory: the
//     packed E2M1 B is expanded on its way in by the TMA unit (16 x 4-bit values into 16
//     bytes, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B).
//
// Every format stages 128-byte shared-memory rows per k-tile and issues four MMAs per k-tile:
// 256 K-elements of 64 per MMA (kind::mxf4nvf4) or 128 of 32 (kind::mxf8f6f4).

#include <cstdint>

namespace blackhole::sm100 {

enum class MmaKind { kMxf4Nvf4, kMxf8f6f4 };

struct Nvfp4Format {
  static constexpr MmaKind Kind = MmaKind::kMxf4Nvf4;
  static constexpr int SfVec = 16;            // elements per scale factor
  static constexpr uint32_t ScaleType = 0;    // instruction-descriptor scale format: UE4M3
  static constexpr int MmaK = 64;             // K-elements per tcgen05.mma
  static constexpr int TileK = 256;           // K-elements per 128-byte shared-memory row
  static constexpr int ABits = 4;             // bits per element in global memory
  static constexpr int BBits = 4;
  static constexpr uint32_t AFormat = 1;      // instruction-descriptor element formats
  static constexpr uint32_t BFormat = 1;      //   (kind::mxf4nvf4: E2M1 = 1)
  static constexpr bool BExpand = false;      // B expanded to a byte per element in smem
};

struct Mxfp4Format {
  static constexpr MmaKind Kind = MmaKind::kMxf4Nvf4;
  static constexpr int SfVec = 32;
  static constexpr uint32_t ScaleType = 1;    // UE8M0
  static constexpr int MmaK = 64;
  static constexpr int TileK = 256;
  static constexpr int ABits = 4;
  static constexpr int BBits = 4;
  static constexpr uint32_t AFormat = 1;
  static constexpr uint32_t BFormat = 1;
  static constexpr bool BExpand = false;
};

struct Mxf8f4Format {
  static constexpr MmaKind Kind = MmaKind::kMxf8f6f4;
  static constexpr int SfVec = 32;
  static constexpr uint32_t ScaleType = 1;    // UE8M0
  static constexpr int MmaK = 32;
  static constexpr int TileK = 128;
  static constexpr int ABits = 8;
  static constexpr int BBits = 4;
  static constexpr uint32_t AFormat = 0;      // kind::mxf8f6f4: E4M3 = 0
  static constexpr uint32_t BFormat = 5;      //                 E2M1 = 5
  static constexpr bool BExpand = true;
};

// Derived per-format constants shared by the schedules.
template <class Fmt>
struct BlockScaleGeometry {
  static constexpr int RowBytes = 128;                         // shared-memory row per k-tile
  static constexpr int KSteps = Fmt::TileK / Fmt::MmaK;        // MMAs per k-tile (4)
  // One 512-byte scale-factor atom holds 4 scales per row, i.e. 4 * SfVec K-elements; the
  // MMAs of k-step j read atom j / StepsPerAtom, starting at byte SfIdStep * (j % StepsPerAtom)
  // of each 4-byte entry (the scale-factor ID).
  static constexpr int StepsPerAtom = 4 * Fmt::SfVec / Fmt::MmaK;   // 1, 2 or 4
  static constexpr int SfIdStep = Fmt::MmaK / Fmt::SfVec;           // scales per MMA: 4, 2, 1
  static constexpr int SfAtoms = KSteps / StepsPerAtom;             // atoms per k-tile: 4, 2, 1
  // global bytes of one row of A / B per k-tile (what a TMA box row transfers)
  static constexpr int ARowTx = Fmt::TileK * Fmt::ABits / 8;        // 128
  static constexpr int BRowTx = Fmt::TileK * Fmt::BBits / 8;        // 128, or 64 expanded
  static_assert(KSteps == 4 && SfAtoms * StepsPerAtom == KSteps, "k-tile geometry");
  static_assert(Fmt::TileK * (Fmt::BExpand ? 8 : Fmt::BBits) / 8 == RowBytes, "B smem row");
  static_assert(Fmt::TileK * Fmt::ABits / 8 == RowBytes, "A smem row");
  static constexpr uint32_t sf_id(int j) { return uint32_t(SfIdStep * (j % StepsPerAtom)); }
};

}  // namespace blackhole::sm100
