#pragma once

// NVFP4 scale-factor layout helpers, host and device.
//
// Scale factors (one UE4M3 byte per 16 K-elements) use the 128x4 blocked layout of
// CUTLASS's Sm1xxBlockScaledConfig, which the reference exposes as make_layout_SFA/SFB
// (include/blackhole/sm120/nvfp4_gemm.hpp:293-298):
//
//   * a 512-byte atom covers 128 rows x 4 K-groups (64 K-elements);
//     inside it, row mn / group kg sits at byte (mn%32)*16 + ((mn/32)%4)*4 + kg%4;
//   * atoms advance along K first (kg/4), then along rows (mn/128).
//
// So the scale factors of one 128-row block for a run of K are one contiguous range,
// which is what lets the kernel fetch them with plain bulk copies.
//
// sf_storage_bytes() returns the layout's full extent (rows padded to 128, K-groups to a
// multiple of 4).  The reference's sf_storage_bytes (nvfp4_gemm.hpp:300-302) returns
// MN*K/16, which is short whenever MN % 128 != 0; callers must allocate this size.

#include <cstdint>

#if defined(__CUDACC__)
#  define BLACKHOLE_HD __host__ __device__
#else
#  define BLACKHOLE_HD
#endif

namespace blackhole {

constexpr int kNvfp4SfVec = 16;    // elements per scale factor
constexpr int kSfAtomRows = 128;   // rows per atom
constexpr int kSfAtomGroups = 4;   // K-groups per atom
constexpr int kSfAtomBytes = 512;  // bytes per atom

// Number of 512-byte atoms along K for a K extent of k elements.
BLACKHOLE_HD constexpr int64_t sf_k_atoms(int64_t k) {
  return (k / kNvfp4SfVec + kSfAtomGroups - 1) / kSfAtomGroups;
}

BLACKHOLE_HD constexpr int64_t sf_offset(int64_t mn, int64_t kg, int64_t k) {
  return ((mn / kSfAtomRows) * sf_k_atoms(k) + kg / kSfAtomGroups) * kSfAtomBytes +
         (mn % 32) * 16 + ((mn / 32) % 4) * 4 + (kg % kSfAtomGroups);
}

BLACKHOLE_HD constexpr int64_t sf_storage_bytes(int64_t mn, int64_t k) {
  return ((mn + kSfAtomRows - 1) / kSfAtomRows) * sf_k_atoms(k) * kSfAtomBytes;
}

// The same layout with `vs`-element K groups (vs = 16: NVFP4; vs = 32: MXFP4, one UE8M0 byte
// per 32 elements -- CUTLASS Sm1xxBlockScaledConfig<32>).  An atom then covers 128 K-elements.
BLACKHOLE_HD constexpr int64_t sf_k_atoms_vs(int64_t k, int vs) {
  return (k / vs + kSfAtomGroups - 1) / kSfAtomGroups;
}
BLACKHOLE_HD constexpr int64_t sf_offset_vs(int64_t mn, int64_t kg, int64_t k, int vs) {
  return ((mn / kSfAtomRows) * sf_k_atoms_vs(k, vs) + kg / kSfAtomGroups) * kSfAtomBytes +
         (mn % 32) * 16 + ((mn / 32) % 4) * 4 + (kg % kSfAtomGroups);
}
BLACKHOLE_HD constexpr int64_t sf_storage_bytes_vs(int64_t mn, int64_t k, int vs) {
  return ((mn + kSfAtomRows - 1) / kSfAtomRows) * sf_k_atoms_vs(k, vs) * kSfAtomBytes;
}

// Byte offset of the atom holding rows [128*row_block, +128) and K-groups [4*k_atom, +4).
BLACKHOLE_HD constexpr int64_t sf_atom_offset(int64_t row_block, int64_t k_atom, int64_t k) {
  return (row_block * sf_k_atoms(k) + k_atom) * kSfAtomBytes;
}

}  // namespace blackhole
