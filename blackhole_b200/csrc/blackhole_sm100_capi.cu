// C ABI of the sm_100a NVFP4 GEMM (declarations: include/blackhole_sm100.h).
// Builds into blackhole_b200/libblackhole_sm100.so; the kernels come from the header-only
// operator in include/blackhole/sm100/.
#include <blackhole_sm100.h>

#include <blackhole/common/sf_layout.hpp>
#include <blackhole/sm100/nvfp4_gemm.hpp>
#include <blackhole/sm100/nvfp4_quant.hpp>
#include <blackhole/sm100/bounded_wait_selftest.hpp>
#include <blackhole/sm100/peer_barrier.hpp>

#include <cstring>
#include <map>
#include <mutex>

// ---------------------------------------------------------------------------------------
// Allocation-free skinny GEMM (blackhole_sm100_nvfp4_bf16_gemm_noalloc).
//
// Some callers cannot allocate device memory at the point where they run the GEMM: serving
// engines that reserve all device memory at start-up and forbid allocation afterwards,
// latency-critical paths that must not pay cudaMalloc's implicit device synchronisation,
// and plugin hosts that hand a plugin nothing but its input and output buffers.  The
// skinny schedule needs scratch (one flag word per epilogue warp and an FP32 partial tile
// per CTA), so this entry point keeps that scratch in a fixed array of this module instead.
//
// The array holds what M <= 16 needs on a device with up to 160 SMs:
//   flags    : 160 CTAs x 8 flag words x 4 bytes + a 4-byte ticket counter, padded to 5376 bytes
//   partials : 160 CTAs x 16 rows x 128 columns x 4 bytes = 1,310,720 bytes
// Every GPU that loads this library holds these 1,316,096 bytes until the process exits.
// ---------------------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxM = 16;
constexpr int kNoAllocMaxSms = 160;
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(
    blackhole::sm100::nvfp4_skinny_workspace_bytes(kNoAllocMaxSms, kNoAllocMaxM));
static_assert(kNoAllocScratchBytes == 1316096, "documented size of the scratch array");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The symbol above names a host-side stand-in, not a device address, so the kernel must be
// given the address that cudaGetSymbolAddress returns for the current device.  Only a
// successful lookup is kept: a first call that fails (for instance one made during a stream
// capture) returns its error and the next call looks the address up again.
struct NoAllocDevice {
  std::mutex mu;
  void* scratch = nullptr;   // non-null once looked up
};

cudaError_t noalloc_scratch(void** out) {
  static NoAllocDevice devs[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  NoAllocDevice& d = devs[dev];
  std::lock_guard<std::mutex> lock(d.mu);
  if (!d.scratch) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    d.scratch = p;
  }
  *out = d.scratch;
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------------
// CUDA IPC for the gathered N-split: a rank exports the allocation holding its output buffer
// and the other ranks map it.  The handle names the whole cudaMalloc allocation, so the
// buffer's offset inside it travels with the handle.
// ---------------------------------------------------------------------------------------
using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = []() -> GetAddressRangeFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<GetAddressRangeFn>(ptr);
  }();
  return fn;
}

std::mutex g_ipc_mu;
std::map<uintptr_t, void*> g_ipc_open;   // pointer handed out -> mapped allocation base

}  // namespace

extern "C" {

int blackhole_sm100_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return static_cast<int>(cudaErrorInvalidValue);
  GetAddressRangeFn range = address_range_fn();
  if (!range) return static_cast<int>(cudaErrorNotSupported);
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return static_cast<int>(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return static_cast<int>(e);
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return 0;
}

int blackhole_sm100_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) return static_cast<int>(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return static_cast<int>(e);
  void* p = static_cast<uint8_t*>(base) + offset;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  g_ipc_open[reinterpret_cast<uintptr_t>(p)] = base;
  *ptr = p;
  return 0;
}

int blackhole_sm100_ipc_close(void* ptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_ipc_mu);
    auto it = g_ipc_open.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == g_ipc_open.end()) return static_cast<int>(cudaErrorInvalidValue);
    base = it->second;
    g_ipc_open.erase(it);
  }
  return static_cast<int>(cudaIpcCloseMemHandle(base));
}

int blackhole_sm100_peer_barrier(void* const* flags, int world, int rank, uint64_t epoch,
                                 uint64_t limit_ns, cudaStream_t stream) {
  return static_cast<int>(
      blackhole::sm100::peer_barrier(flags, world, rank, epoch, limit_ns, stream));
}

int blackhole_sm100_nvfp4_bf16_gemm_gather(int M, int N, int K, const void* A, const void* SFA,
                                           const void* B, const void* SFB, void* const* dst,
                                           int ndst, int64_t col0, int64_t ldd, float alpha,
                                           cudaStream_t stream) {
  return static_cast<int>(blackhole::sm100::nvfp4_bf16_gemm_gather(
      M, N, K, A, SFA, B, SFB, dst, ndst, col0, ldd, alpha, stream));
}

int blackhole_sm100_nvfp4_bf16_gemm(int M, int N, int K, const void* A, const void* SFA,
                                    const void* B, const void* SFB, void* D, float alpha,
                                    cudaStream_t stream) {
  return static_cast<int>(
      blackhole::sm100::nvfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha, stream));
}

int blackhole_sm100_nvfp4_bf16_gemm_ex(int M, int N, int K, const void* A, const void* SFA,
                                       const void* B, const void* SFB, void* D, float alpha,
                                       int schedule, void* workspace, int64_t workspace_bytes,
                                       cudaStream_t stream) {
  if (schedule < 0 || schedule > 4) return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(blackhole::sm100::nvfp4_bf16_gemm_ex(
      M, N, K, A, SFA, B, SFB, D, alpha, static_cast<blackhole::sm100::Nvfp4Schedule>(schedule),
      workspace, workspace_bytes, stream));
}

int blackhole_sm100_mxfp4_bf16_gemm(int M, int N, int K, const void* A, const void* SFA,
                                    const void* B, const void* SFB, void* D, float alpha,
                                    cudaStream_t stream) {
  return static_cast<int>(
      blackhole::sm100::mxfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha, stream));
}

int blackhole_sm100_mxfp4_bf16_gemm_ex(int M, int N, int K, const void* A, const void* SFA,
                                       const void* B, const void* SFB, void* D, float alpha,
                                       int schedule, void* workspace, int64_t workspace_bytes,
                                       cudaStream_t stream) {
  if (schedule < 0 || schedule > 4) return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(blackhole::sm100::mxfp4_bf16_gemm_ex(
      M, N, K, A, SFA, B, SFB, D, alpha, static_cast<blackhole::sm100::Nvfp4Schedule>(schedule),
      workspace, workspace_bytes, stream));
}

int blackhole_sm100_mxf8f4_bf16_gemm(int M, int N, int K, const void* A, const void* SFA,
                                     const void* B, const void* SFB, void* D, float alpha,
                                     cudaStream_t stream) {
  return static_cast<int>(blackhole::sm100::mxf8f4_bf16_gemm_ex(
      M, N, K, A, SFA, B, SFB, D, alpha, blackhole::sm100::Nvfp4Schedule::kAuto, nullptr, 0,
      stream));
}

int blackhole_sm100_mxf8f4_bf16_gemm_ex(int M, int N, int K, const void* A, const void* SFA,
                                        const void* B, const void* SFB, void* D, float alpha,
                                        int schedule, void* workspace, int64_t workspace_bytes,
                                        cudaStream_t stream) {
  if (schedule < 0 || schedule > 4) return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(blackhole::sm100::mxf8f4_bf16_gemm_ex(
      M, N, K, A, SFA, B, SFB, D, alpha, static_cast<blackhole::sm100::Nvfp4Schedule>(schedule),
      workspace, workspace_bytes, stream));
}

int blackhole_sm100_mxfp8_quantize(const void* X, int x_is_bf16, int rows, int K, void* q,
                                   void* sf, cudaStream_t stream) {
  return static_cast<int>(
      blackhole::sm100::mxfp8_quantize(X, x_is_bf16, rows, K, q, sf, stream));
}

int64_t blackhole_sm100_mxfp4_sf_storage_bytes(int64_t mn, int64_t k) {
  if (mn < 0 || k < 0) return -1;
  return blackhole::sf_storage_bytes_vs(mn, k, 32);
}

int blackhole_sm100_mxfp4_quantize(const void* X, int x_is_bf16, int rows, int K, void* packed,
                                   void* sf, cudaStream_t stream) {
  return static_cast<int>(
      blackhole::sm100::mxfp4_quantize(X, x_is_bf16, rows, K, packed, sf, stream));
}

int64_t blackhole_sm100_workspace_bytes(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 1) return -1;
  if (M > 128) return 0;
  blackhole::sm100::detail::DeviceState* st = blackhole::sm100::detail::prepare_device();
  if (!st || st->init_err != cudaSuccess) return -1;
  return blackhole::sm100::nvfp4_skinny_workspace_bytes(st->num_sms,
                                                       blackhole::sm100::nvfp4_skinny_mpad(M));
}

int64_t blackhole_sm100_sf_storage_bytes(int64_t mn, int64_t k) {
  if (mn < 0 || k < 0) return -1;
  return blackhole::sf_storage_bytes(mn, k);
}

int64_t blackhole_sm100_sf_offset(int64_t mn, int64_t kg, int64_t k) {
  if (mn < 0 || kg < 0 || k < 0) return -1;
  return blackhole::sf_offset(mn, kg, k);
}

int blackhole_sm100_device_status(int device, unsigned int* status, int clear) {
  if (!status) return static_cast<int>(cudaErrorInvalidValue);
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = blackhole::sm100::read_device_status(status, clear != 0);
  cudaSetDevice(prev);
  return static_cast<int>(e);
}

int blackhole_sm100_nvfp4_quantize(const void* X, int x_is_bf16, int rows, int K, void* packed,
                                   void* sf, float* scales, cudaStream_t stream) {
  return static_cast<int>(
      blackhole::sm100::nvfp4_quantize(X, x_is_bf16, rows, K, packed, sf, scales, stream));
}

int blackhole_sm100_nvfp4_bf16_gemm_noalloc(int M, int N, int K, const void* A, const void* SFA,
                                            const void* B, const void* SFB, void* D, float alpha,
                                            cudaStream_t stream) {
  cudaError_t e = blackhole::sm100::nvfp4_check_args(M, N, K, A, SFA, B, SFB, D);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (M > kNoAllocMaxM) return static_cast<int>(cudaErrorInvalidValue);  // beyond the array
  blackhole::sm100::detail::DeviceState* st = blackhole::sm100::detail::prepare_device();
  if (!st) return static_cast<int>(cudaErrorInvalidDevice);
  if (st->init_err != cudaSuccess) return static_cast<int>(st->init_err);
  const int64_t need = blackhole::sm100::nvfp4_skinny_workspace_bytes(
      st->num_sms, blackhole::sm100::nvfp4_skinny_mpad(M));
  if (st->num_sms > kNoAllocMaxSms || need > static_cast<int64_t>(kNoAllocScratchBytes))
    return static_cast<int>(cudaErrorInvalidValue);
  void* scratch = nullptr;
  e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  // The array keeps whatever the previous call left; the flag words must start at zero.
  e = cudaMemsetAsync(scratch, 0,
                      static_cast<size_t>(blackhole::sm100::nvfp4_skinny_flag_bytes(st->num_sms)),
                      stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(blackhole::sm100::nvfp4_bf16_gemm_skinny(
      M, N, K, A, SFA, B, SFB, D, alpha, scratch, static_cast<int64_t>(kNoAllocScratchBytes),
      stream));
}

int blackhole_sm100_selftest_skinny_partial_wait(int M, int N, int K, const void* A,
                                                 const void* SFA, const void* B, const void* SFB,
                                                 void* D, float alpha, void* workspace,
                                                 int64_t workspace_bytes, uint64_t partial_wait_ns,
                                                 cudaStream_t stream) {
  if (partial_wait_ns == 0 || partial_wait_ns > blackhole::sm100::ptx::kWaitLimitNs || M > 128)
    return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(blackhole::sm100::block_scaled_bf16_gemm_skinny<
                          blackhole::sm100::Nvfp4Format>(
      M, N, K, A, SFA, B, SFB, D, alpha, workspace, workspace_bytes, stream, 1 << 30, true,
      nullptr, partial_wait_ns));
}

int blackhole_sm100_selftest_bounded_wait(uint64_t limit_ns, uint64_t* result,
                                          cudaStream_t stream) {
  return static_cast<int>(blackhole::sm100::bounded_wait_selftest(limit_ns, result, stream));
}

int blackhole_sm100_abi_version(void) { return BLACKHOLE_SM100_ABI_VERSION; }

}  // extern "C"
