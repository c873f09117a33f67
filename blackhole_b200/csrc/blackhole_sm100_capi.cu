// C ABI of the sm_100a NVFP4 GEMM (declarations: include/blackhole_sm100.h).
// Builds into blackhole_b200/libblackhole_sm100.so; the kernels come from the header-only
// operator in include/blackhole/sm100/.
#include <blackhole_sm100.h>

#include <blackhole/common/sf_layout.hpp>
#include <blackhole/sm100/nvfp4_gemm.hpp>
#include <blackhole/sm100/nvfp4_quant.hpp>

extern "C" {

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
  if (schedule < 0 || schedule > 3) return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(blackhole::sm100::nvfp4_bf16_gemm_ex(
      M, N, K, A, SFA, B, SFB, D, alpha, static_cast<blackhole::sm100::Nvfp4Schedule>(schedule),
      workspace, workspace_bytes, stream));
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

int blackhole_sm100_abi_version(void) { return BLACKHOLE_SM100_ABI_VERSION; }

}  // extern "C"
