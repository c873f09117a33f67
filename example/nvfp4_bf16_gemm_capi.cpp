// The example built by a host C++ compiler: without nvcc, <blackhole/sm100/nvfp4_gemm.hpp>
// forwards blackhole::sm100::nvfp4_bf16_gemm to the C ABI of libblackhole_sm100.so
// (include/blackhole_sm100.h), so this program links that library and the CUDA runtime only.
#include "nvfp4_bf16_gemm.cu"
