#pragma once

// Shared host/device pieces of the sm_100a NVFP4 GEMM schedules: argument checks, status
// word, tensor-map encoding and per-device state.

#include <cstddef>
#include <cstdint>
#include <type_traits>

#include <cuda_runtime_api.h>

#include <blackhole/common/arch.hpp>
#include <blackhole/common/sf_layout.hpp>

#if defined(__CUDACC__)
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include <blackhole/sm100/ptx.hpp>
#endif

namespace blackhole::sm100 {

// Gather mode (the N-split's all-gather fused into the GEMM): besides this GPU's buffer, up to
// kMaxGatherPeers further buffers (the other GPUs of an eight-GPU node) receive every tile.
constexpr int kMaxGatherPeers = 7;

// Status bits written when a bounded wait gives up.
enum : uint32_t {
  kStatusLoadTimeout = 1u,
  kStatusMmaTimeout = 2u,
  kStatusEpilogueTimeout = 4u,
  kStatusBarrierTimeout = 8u,     // peer_barrier: a peer's signal did not arrive in time
};

// Shape / alignment check shared by every schedule and the C ABI (host only, no CUDA calls).
// The reference accepts M % 128 == 0, N % 128 == 0, K % 256 == 0 (nvfp4_gemm.hpp:594-596);
// here any M >= 1, N % 8 == 0 and K % 32 == 0 are accepted (tiles past M / N / K read zeros
// through TMA and are clipped on store; N % 8 keeps D's rows and K % 32 the packed rows of A
// and B 16-byte aligned for TMA).
inline cudaError_t nvfp4_check_args(int M, int N, int K, const void* A, const void* SFA,
                                    const void* B, const void* SFB, const void* D) {
  if (M < 1 || N < 8 || K < 32) return cudaErrorInvalidValue;
  if (N % 8 != 0 || K % 32 != 0) return cudaErrorInvalidValue;
  if (!A || !SFA || !B || !SFB || !D) return cudaErrorInvalidValue;
  auto mis = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (mis(A) || mis(SFA) || mis(B) || mis(SFB) || mis(D)) return cudaErrorInvalidValue;
  if (static_cast<int64_t>(M) * N > (int64_t(1) << 46)) return cudaErrorInvalidValue;
  return cudaSuccess;
}

#if defined(__CUDACC__)

namespace detail {

// Destinations of a gather-mode call: dst[0] is this GPU's buffer, dst[1..ndst) further
// buffers written with plain stores; every buffer is row-major with rows ldd elements apart
// and receives the call's M x N result at columns [col0, col0 + N).
struct GatherSpec {
  void* const* dst;
  int ndst;
  int64_t col0;
  int64_t ldd;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Bounded wait used only on the abort path: does not look at the abort flag.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer_ns() - t0 > 200000000ull) break;
  }
}

static __device__ uint32_t g_status;  // or-ed status bits of this module's kernels

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// Encoding a tensor map costs microseconds on the host, comparable to a decode-sized GEMM,
// so encoded maps are kept in a small per-thread cache keyed by everything they encode
// (kind, base address, extents, box).  A map holds no reference to the memory, so a hit
// after the buffer was freed and another allocated at the same address is still correct.
struct TmapKey {
  int kind;
  const void* base;
  int64_t a, b;
  uint32_t c, d;
  bool operator==(const TmapKey& o) const {
    return kind == o.kind && base == o.base && a == o.a && b == o.b && c == o.c && d == o.d;
  }
};

template <class Make>
inline cudaError_t cached_tmap(const TmapKey& key, CUtensorMap* out, Make make) {
  struct Entry {
    TmapKey key;
    CUtensorMap map;
    bool valid = false;
  };
  constexpr int kEntries = 16;
  thread_local Entry cache[kEntries];
  thread_local int next = 0;
  for (int i = 0; i < kEntries; ++i) {
    if (cache[i].valid && cache[i].key == key) {
      *out = cache[i].map;
      return cudaSuccess;
    }
  }
  cudaError_t e = make(out);
  if (e != cudaSuccess) return e;
  Entry& slot = cache[next];
  next = (next + 1) % kEntries;
  slot.key = key;
  slot.map = *out;
  slot.valid = true;
  return cudaSuccess;
}

// 2-D K-major byte tensor [rows][row_bytes] with a (box_rows x box_bytes) box swizzled at
// box_bytes (128, 64 or 32).  Rows past `rows` read as zero.
inline cudaError_t make_kmajor_tmap_uncached(CUtensorMap* m, const void* base, int64_t rows,
                                             int64_t row_bytes, uint32_t box_rows,
                                             uint32_t box_bytes) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {box_bytes, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapSwizzle swz = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                   : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Scale factors viewed as rows of 512-byte atoms (64 x 8 bytes): [row_blocks * k_atoms][64].
// A box of box_atoms atoms is one (64 * box_atoms)-wide k-tile of one 128-row block; atoms
// past the end (row blocks beyond the tensor) read as zero.
inline cudaError_t make_sf_tmap_uncached(CUtensorMap* m, const void* base, int64_t mn, int64_t k,
                                         uint32_t box_atoms) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  const int64_t atoms = ((mn + 127) / 128) * sf_k_atoms(k);
  cuuint64_t dims[2] = {64u, static_cast<cuuint64_t>(atoms)};
  cuuint64_t strides[1] = {512u};
  cuuint32_t box[2] = {64u, box_atoms};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Scale factors of one operand as a 3-D tensor [row blocks][k-tiles][2048 B]: the 4 atoms of
// one 128-row block and one 256-wide k-tile are 2 KB contiguous.  A box of {2048 B, ktiles,
// blocks} fetches `ktiles` k-tiles of `blocks` consecutive row blocks in one request, as
// 2 KB rows, landing as [block][k-tile][2048 B]; parts past the edge read zeros.  (Measured
// on B200: every scale-factor request in flight slows the two-SM schedule's tensor pipe, far
// beyond its bytes, so they are made few and long.)
inline cudaError_t make_sf_tmap_ktile_uncached(CUtensorMap* m, const void* base, int64_t mn,
                                               int64_t k, uint32_t blocks, uint32_t ktiles,
                                               int atoms_per_ktile, int vs) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  const int64_t k_atoms = sf_k_atoms_vs(k, vs);
  if (k_atoms % atoms_per_ktile != 0) return cudaErrorInvalidValue;
  const uint32_t row_words = 64u * uint32_t(atoms_per_ktile);   // 8-byte elements per row
  cuuint64_t dims[3] = {row_words, static_cast<cuuint64_t>(k_atoms / atoms_per_ktile),
                        static_cast<cuuint64_t>((mn + 127) / 128)};
  cuuint64_t strides[2] = {row_words * 8u, static_cast<cuuint64_t>(k_atoms * 512)};
  cuuint32_t box[3] = {row_words, ktiles, blocks};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Scale factors as a 3-D tensor [row blocks][atoms][512 B] for K % 256 != 0: a box of
// {512 B, 4 atoms, blocks} lands as [block][atom][512 B], the same layout as the k-tile map,
// and atoms past the last one of a block (the K tail) read zeros instead of running into the
// next block or past the end of the buffer.
inline cudaError_t make_sf_tmap_atoms_uncached(CUtensorMap* m, const void* base, int64_t mn,
                                               int64_t k, uint32_t blocks, uint32_t atoms,
                                               int vs) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  const int64_t k_atoms = sf_k_atoms_vs(k, vs);
  cuuint64_t dims[3] = {64u, static_cast<cuuint64_t>(k_atoms),
                        static_cast<cuuint64_t>((mn + 127) / 128)};
  cuuint64_t strides[2] = {512u, static_cast<cuuint64_t>(k_atoms * 512)};
  cuuint32_t box[3] = {64u, atoms, blocks};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Row-major BF16 [rows][cols] output with a (32 rows x box_cols columns) box: the store box
// of one epilogue warp.  Parts of a box past the tensor edge are not written.
// box_cols = 64 (128-byte rows, 128B swizzle) or 16 (32-byte rows, 32B swizzle).
// ld: elements between consecutive rows (>= cols; 0 means cols).
inline cudaError_t make_d_tmap_uncached(CUtensorMap* m, void* base, int64_t rows, int64_t cols,
                                        uint32_t box_cols, int64_t ld = 0) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>((ld > 0 ? ld : cols) * 2)};
  cuuint32_t box[2] = {box_cols, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapSwizzle swz = box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

inline cudaError_t make_kmajor_tmap(CUtensorMap* m, const void* base, int64_t rows,
                                    int64_t row_bytes, uint32_t box_rows, uint32_t box_bytes = 128) {
  return cached_tmap({0, base, rows, row_bytes, box_rows, box_bytes}, m, [&](CUtensorMap* o) {
    return make_kmajor_tmap_uncached(o, base, rows, row_bytes, box_rows, box_bytes);
  });
}
// Packed 4-bit [rows][K] operand read as CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B: every 16
// values (8 bytes) land in 16 bytes of shared memory, the one-byte-per-element form
// kind::mxf8f6f4 reads.  Box: 128 elements (a 128-byte smem row, 128B swizzle) x box_rows;
// x coordinates are in elements.  Needs K % 128 == 0 and a 32-byte aligned base.
inline cudaError_t make_fp4_expand_tmap_uncached(CUtensorMap* m, const void* base, int64_t rows,
                                                 int64_t k, uint32_t box_rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k / 2)};
  cuuint32_t box[2] = {128u, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}
inline cudaError_t make_fp4_expand_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t k,
                                        uint32_t box_rows) {
  return cached_tmap({6, base, rows, k, box_rows, 0}, m, [&](CUtensorMap* o) {
    return make_fp4_expand_tmap_uncached(o, base, rows, k, box_rows);
  });
}
// Operand maps of a format: 128-byte boxes of box_rows rows per k-tile.
template <class Fmt>
inline cudaError_t make_a_tmap(CUtensorMap* m, const void* A, int64_t rows, int64_t k,
                               uint32_t box_rows) {
  return make_kmajor_tmap(m, A, rows, k * Fmt::ABits / 8, box_rows);
}
template <class Fmt>
inline cudaError_t make_b_tmap(CUtensorMap* m, const void* B, int64_t rows, int64_t k,
                               uint32_t box_rows) {
  if constexpr (Fmt::BExpand)
    return make_fp4_expand_tmap(m, B, rows, k, box_rows);
  else
    return make_kmajor_tmap(m, B, rows, k * Fmt::BBits / 8, box_rows);
}
// Shapes and alignment a format adds to nvfp4_check_args: the expanded 4-bit B needs
// K % 128 == 0 (a whole k-tile) and a 32-byte aligned base.
template <class Fmt>
inline cudaError_t format_check_args(int K, const void* B) {
  if constexpr (Fmt::BExpand) {
    if (K % 128 != 0 || (reinterpret_cast<uintptr_t>(B) & 31u)) return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}
inline cudaError_t make_sf_tmap(CUtensorMap* m, const void* base, int64_t mn, int64_t k,
                                uint32_t box_atoms = 4) {
  return cached_tmap({1, base, mn, k, box_atoms, 0}, m, [&](CUtensorMap* o) {
    return make_sf_tmap_uncached(o, base, mn, k, box_atoms);
  });
}
inline cudaError_t make_sf_tmap_ktile(CUtensorMap* m, const void* base, int64_t mn, int64_t k,
                                      uint32_t blocks, uint32_t ktiles, int atoms_per_ktile = 4,
                                      int vs = 16) {
  return cached_tmap({3 + 16 * vs + 256 * atoms_per_ktile, base, mn, k, blocks, ktiles}, m,
                     [&](CUtensorMap* o) {
                       return make_sf_tmap_ktile_uncached(o, base, mn, k, blocks, ktiles,
                                                          atoms_per_ktile, vs);
                     });
}
inline cudaError_t make_sf_tmap_atoms(CUtensorMap* m, const void* base, int64_t mn, int64_t k,
                                      uint32_t blocks, uint32_t atoms = 4, int vs = 16) {
  return cached_tmap({4 + 16 * vs, base, mn, k, blocks, atoms}, m, [&](CUtensorMap* o) {
    return make_sf_tmap_atoms_uncached(o, base, mn, k, blocks, atoms, vs);
  });
}
inline cudaError_t make_d_tmap(CUtensorMap* m, void* base, int64_t rows, int64_t cols,
                               uint32_t box_cols = 64, int64_t ld = 0) {
  return cached_tmap({2, base, rows, cols, box_cols, static_cast<uint32_t>(ld)}, m,
                     [&](CUtensorMap* o) {
                       return make_d_tmap_uncached(o, base, rows, cols, box_cols, ld);
                     });
}

struct DeviceState {
  std::mutex mu;
  bool ready = false;               // set once, under mu, after a successful set-up
  cudaError_t init_err = cudaSuccess;
  int num_sms = 0;
  uint32_t* status = nullptr;
};

inline DeviceState& device_state(int dev) {
  static DeviceState states[64];
  return states[dev & 63];
}

// Per-device set-up (the reference keeps a process-wide static bool instead,
// nvfp4_gemm.hpp:625-631, which misses every device after the first).  Only a successful
// set-up is kept: after a failure (for instance a first call made while the stream is being
// captured, where cudaGetSymbolAddress is not allowed) the returned state carries the error
// and the next call tries again.
inline DeviceState* prepare_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  // The tensor-map encoder is a driver call and needs a context current on this host thread.
  // A thread whose only CUDA calls so far were ones that bind none (cudaGetDevice, cached
  // set-up) has none, and the encoder then fails (seen: a new thread's first one-SM call after
  // another thread had done the per-device set-up).  cudaFree(nullptr) does nothing but make
  // the runtime bind the device's primary context, or keep the one the thread already has;
  // once per thread and device.
  thread_local uint64_t bound = 0;
  if (!(bound & (uint64_t(1) << dev))) {
    e = cudaFree(nullptr);
    if (e != cudaSuccess) {
      thread_local DeviceState unbound;
      unbound.init_err = e;
      return &unbound;
    }
    bound |= uint64_t(1) << dev;
  }
  DeviceState& st = device_state(dev);
  std::lock_guard<std::mutex> lock(st.mu);
  if (st.ready) return &st;
  int sms = 0;
  void* sym = nullptr;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&sym, g_status);
  if (e != cudaSuccess) {
    thread_local DeviceState failed;   // this call's error; the shared state stays unset
    failed.init_err = e;
    return &failed;
  }
  st.num_sms = sms;
  st.status = static_cast<uint32_t*>(sym);
  st.init_err = cudaSuccess;
  st.ready = true;
  return &st;
}

// Sets a kernel's dynamic shared-memory limit once per (device, kernel function).
template <class Kernel>
inline cudaError_t set_smem_once(Kernel kernel, int bytes, int dev) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, cudaError_t> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  done[key] = e;
  return e;
}

// Launches with programmatic stream serialization, so the kernel may start while the
// previous kernel in the stream drains (the kernels call pdl_wait_prior_grid() before they
// touch global memory).
template <class Params>
inline cudaError_t launch_pdl(void (*kernel)(Params), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace detail

// Reads (and optionally clears) the status word of this module on the current device.
inline cudaError_t read_device_status(unsigned int* out, bool clear) {
  detail::DeviceState* st = detail::prepare_device();
  if (!st) return cudaErrorInvalidDevice;
  if (st->init_err != cudaSuccess) return st->init_err;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(out, detail::g_status, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  if (clear) {
    unsigned int z = 0;
    e = cudaMemcpyToSymbol(detail::g_status, &z, sizeof(unsigned int));
  }
  return e;
}

#endif  // __CUDACC__

}  // namespace blackhole::sm100
