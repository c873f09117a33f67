/*
 * blackhole_sm100.h -- C ABI of the B200 (sm_100a) NVFP4 x NVFP4 -> BF16 GEMM.
 *
 * Exported by blackhole_b200/libblackhole_sm100.so.  Plain pointers and sizes only; every
 * buffer is caller-owned device memory and every call is asynchronous on `stream`.
 * Return values are cudaError_t codes (0 = cudaSuccess).
 */
#ifndef BLACKHOLE_SM100_H
#define BLACKHOLE_SM100_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BLACKHOLE_SM100_ABI_VERSION 6

#if defined(__GNUC__)
#define BLACKHOLE_SM100_API __attribute__((visibility("default")))
#else
#define BLACKHOLE_SM100_API
#endif

/* D = bf16(alpha * A . B^T), block-scaled NVFP4 operands.
 *
 * Replaces blackhole::sm120::nvfp4_bf16_gemm(M, N, K, A_packed, SFA, B_packed, SFB, D,
 * stream) of the reference (include/blackhole/sm120/nvfp4_gemm.hpp:588-591); the argument
 * meanings are the reference's (nvfp4_gemm.hpp:583-587):
 *   A   : E2M1, M x K, K-contiguous, two per byte, even k in the low nibble
 *   SFA : UE4M3 scale factors of A in the 128x4 blocked layout (make_layout_SFA(M, K))
 *   B   : E2M1, N x K, K-contiguous
 *   SFB : UE4M3 scale factors of B (make_layout_SFB(N, K))
 *   D   : BF16, M x N, row-major
 * plus `alpha`, the product of the two global scales (alpha = 1 reproduces the reference).
 * Shapes: M >= 1, N % 8 == 0, K % 32 == 0 (the reference needs M % 128 == 0, N % 128 == 0
 * and K % 256 == 0).  With K % 64 != 0, the padding scale factors of the last K-groups must be
 * finite (this library's quantiser writes zeros there).
 * SFA/SFB must span blackhole_sm100_sf_storage_bytes(M|N, K) bytes (rows padded to 128).
 * Pointers must be 16-byte aligned.  Errors: cudaErrorInvalidValue for a bad shape,
 * null or misaligned pointer; otherwise the launch status, as in nvfp4_gemm.hpp:594-636.
 * Stream-ordered.  The kernels are launched as programmatic dependents of the previous kernel
 * in the stream: they set up while it finishes, and for M <= 16 also prefetch their first B /
 * SFB tiles into L2 (a cache hint only), but read and write nothing before it completes.
 * By shape: M <= 16 the skinny stream-K schedule, M <= 256 the one-SM, larger M the two-SM. */
BLACKHOLE_SM100_API int blackhole_sm100_nvfp4_bf16_gemm(int M, int N, int K, const void* A, const void* SFA,
                                    const void* B, const void* SFB, void* D, float alpha,
                                    cudaStream_t stream);

/* Same GEMM with an explicit schedule and workspace (no counterpart in the reference, which
 * has a single schedule).  schedule: 0 = by shape (as above), 1 = one-SM 128x256 tiles,
 * 2 = two-SM 256x256 tiles (cta_group::2), 3 = skinny-M stream-K (M <= 128),
 * 4 = skinny-M stream-K without the early L2 prefetch (same results).
 * workspace: device memory for the skinny schedule, at least
 * blackhole_sm100_workspace_bytes(M, N, K) bytes, zero-filled before its first use; every
 * call leaves it ready for the next, a call that gave up on a bounded wait included; NULL
 * selects a library-owned buffer per (device, stream), allocated on first use.  Calls that
 * share one workspace must be ordered (same stream). */
BLACKHOLE_SM100_API int blackhole_sm100_nvfp4_bf16_gemm_ex(int M, int N, int K, const void* A,
                                                           const void* SFA, const void* B,
                                                           const void* SFB, void* D, float alpha,
                                                           int schedule, void* workspace,
                                                           int64_t workspace_bytes,
                                                           cudaStream_t stream);

/* Workspace bytes blackhole_sm100_nvfp4_bf16_gemm_ex needs for this shape on the current
 * device (0 when the shape does not use the skinny schedule); negative on error. */
BLACKHOLE_SM100_API int64_t blackhole_sm100_workspace_bytes(int M, int N, int K);

/* Bytes of a (mn x k) scale-factor tensor in the 128x4 layout, padding included
 * (the cosize of make_layout_SFA/SFB; nvfp4_gemm.hpp:293-302). */
BLACKHOLE_SM100_API int64_t blackhole_sm100_sf_storage_bytes(int64_t mn, int64_t k);

/* Byte offset of the scale factor of row mn, K-group kg (= k/16) for K extent k
 * (make_layout_SFA(M, K)(mn, kg*16); nvfp4_gemm.hpp:293-298). */
BLACKHOLE_SM100_API int64_t blackhole_sm100_sf_offset(int64_t mn, int64_t kg, int64_t k);

/* Device-side status of the calling process's kernels on `device`: nonzero when a kernel
 * gave up on a bounded wait (bit 0: load pipeline, bit 1: MMA pipeline, bit 2: epilogue).
 * Synchronises the device.  With clear != 0 the word is reset afterwards.  The reference
 * has no counterpart (its kernel cannot time out). */
BLACKHOLE_SM100_API int blackhole_sm100_device_status(int device, unsigned int* status, int clear);

/* NVFP4 quantiser: X (rows x K, FP32 when x_is_bf16 == 0, else BF16, K-contiguous,
 * K % 16 == 0) -> packed E2M1 (rows*K/2 bytes), UE4M3 scale factors in the 128x4 layout
 * (sf_storage_bytes(rows, K) bytes, padding written as 0) and scales[0] = amax,
 * scales[1] = global scale g = amax/(448*6) (device float[2]).  Per 16-block:
 * s = UE4M3((amax_b/6)/g), q = E2M1(x/(s*g)), all round-to-nearest-even; alpha of a GEMM
 * is gA*gB.  Device counterpart of the reference example's host quantisation
 * (example/nvfp4_bf16_gemm.cu:60-71, :104-133), following the BASELINE recipe. */
BLACKHOLE_SM100_API int blackhole_sm100_nvfp4_quantize(const void* X, int x_is_bf16, int rows, int K,
                                                       void* packed, void* sf, float* scales,
                                                       cudaStream_t stream);

/* Allocation-free variant of the GEMM for M <= 16 (no counterpart in the reference).
 * For callers that may not allocate device memory when they run the GEMM (memory planned
 * up front, no cudaMalloc synchronisation allowed on the path, or a host that passes only
 * the input and output buffers).  It runs the skinny schedule with its scratch held in a
 * fixed 1,316,096-byte array inside this library, sized for M <= 16 on devices with at most
 * 160 SMs; larger M or more SMs return cudaErrorInvalidValue.  It calls no cudaMalloc or
 * cudaFree.  The first call on each device looks up the array's device address with
 * cudaGetSymbolAddress; make that first call before any stream capture (a lookup that fails,
 * inside a capture for instance, is not kept: the next call tries again).  Every call uses the
 * same array and clears its flag words first (cudaMemsetAsync on `stream`), so calls that
 * overlap on the GPU (different streams, or different host threads) race with each other. */
BLACKHOLE_SM100_API int blackhole_sm100_nvfp4_bf16_gemm_noalloc(int M, int N, int K, const void* A,
                                                                const void* SFA, const void* B,
                                                                const void* SFB, void* D,
                                                                float alpha, cudaStream_t stream);

/* GEMM with the N-split's all-gather fused in (no counterpart in the reference, whose
 * multi-GPU path is the caller's NCCL all-gather of [P][M][N/P] slices): the M x N result goes
 * to columns [col0, col0 + N) of each of the ndst row-major BF16 buffers dst[0..ndst), rows
 * ldd elements apart.  dst[0] must be this GPU's memory; dst[1..] are written tile by tile with
 * plain stores while later tiles compute -- other GPUs' buffers mapped with
 * blackhole_sm100_ipc_open, or local memory.  M <= 128 runs the skinny (decode) schedule, larger
 * M the two-SM schedule.  1 <= ndst <= 8, col0 % 8 == 0,
 * ldd % 8 == 0, col0 + N <= ldd, all dst 16-byte aligned; shapes as blackhole_sm100_nvfp4_bf16_gemm.
 * Asynchronous on `stream`; nothing orders it against other GPUs: the caller synchronises the
 * ranks after the call (e.g. blackhole_sm100_peer_barrier on the same stream) before any rank
 * reads its buffer, and before a call overwrites a buffer another rank may still read. */
BLACKHOLE_SM100_API int blackhole_sm100_nvfp4_bf16_gemm_gather(int M, int N, int K, const void* A,
                                                               const void* SFA, const void* B,
                                                               const void* SFB, void* const* dst,
                                                               int ndst, int64_t col0, int64_t ldd,
                                                               float alpha, cudaStream_t stream);

/* CUDA IPC for those buffers (no counterpart in the reference).  get_handle writes the
 * 64-byte cudaIpcMemHandle_t of the cudaMalloc allocation that holds ptr, and ptr's offset
 * inside it; open maps such a handle from another process on this device and returns the
 * mapped address of the same byte (peer access enabled); close unmaps a pointer open returned. */
BLACKHOLE_SM100_API int blackhole_sm100_ipc_get_handle(const void* ptr, void* handle,
                                                       int64_t* offset);
BLACKHOLE_SM100_API int blackhole_sm100_ipc_open(const void* handle, int64_t offset, void** ptr);
BLACKHOLE_SM100_API int blackhole_sm100_ipc_close(void* ptr);

/* Stream-ordered barrier across the ranks of a gathered N-split (no counterpart in the
 * reference, whose gather is NCCL's).  flags[q] is rank q's array of `world` 64-bit words
 * (zero before the first call, 8-byte aligned) as mapped in this process, flags[rank] this
 * GPU's own; epoch is 1 on the first call and one more on each later call.  Stores epoch with
 * a system-scope release into this rank's word of every peer's array after everything earlier
 * on `stream`, then waits until every peer's word in this GPU's array has reached epoch, so
 * work after it on `stream` sees every rank's gathered tiles.  The wait is bounded by limit_ns
 * (0 < limit_ns <= 1e10): on timeout it sets status bit 8 (blackhole_sm100_device_status) and
 * returns.  1 <= world <= 8; one call per GPU per step (the ranks wait on one another). */
BLACKHOLE_SM100_API int blackhole_sm100_peer_barrier(void* const* flags, int world, int rank,
                                                     uint64_t epoch, uint64_t limit_ns,
                                                     cudaStream_t stream);

/* Self-test of the bounded-wait protocol (no counterpart in the reference): one CTA whose
 * "producer" warp waits limit_ns on a barrier nothing arrives on, gives up, raises the CTA
 * abort flag and sets status bit 0; its "consumer" warp, holding TMEM, must leave through
 * the abort flag (bit 1 stays clear) and free its TMEM.  result: 4 device uint64 words
 * (completed flags of the two warps, then their wait times in ns).  0 < limit_ns <= 2e9.
 * Asynchronous on `stream`; read the status with blackhole_sm100_device_status. */
BLACKHOLE_SM100_API int blackhole_sm100_selftest_bounded_wait(uint64_t limit_ns, uint64_t* result,
                                                              cudaStream_t stream);

/* Self-test hook of the skinny schedule's recovery (no counterpart in the reference): the
 * NVFP4 GEMM on the skinny schedule with a caller workspace, as blackhole_sm100_nvfp4_bf16_gemm_ex
 * with schedule 3, except that a finishing CTA waits at most partial_wait_ns
 * (0 < partial_wait_ns <= 4e9) for the partial sums of the CTAs sharing its row block.  With a
 * bound far below a launch's duration the finishers give up: status bit 2 is set, their
 * output rows are left unwritten and flags of the workspace stay raised.  The next launch on
 * the same workspace must still compute the right result (the flags carry a per-launch tag):
 * tests/test_bounded_wait_gpu.py checks that, without faulting anything. */
BLACKHOLE_SM100_API int blackhole_sm100_selftest_skinny_partial_wait(
    int M, int N, int K, const void* A, const void* SFA, const void* B, const void* SFB, void* D,
    float alpha, void* workspace, int64_t workspace_bytes, uint64_t partial_wait_ns,
    cudaStream_t stream);

/* MXFP4 x MXFP4 -> BF16 (OCP Microscaling v1.0: E2M1 elements, one UE8M0 scale per 32
 * elements along K, in the same 128x4 blocked layout with 32-element groups).  No
 * counterpart in the reference, which serves NVFP4 only: the sibling format behind the same
 * operator shape.  Arguments, shapes, ordering and errors as blackhole_sm100_nvfp4_bf16_gemm;
 * SFA / SFB span blackhole_sm100_mxfp4_sf_storage_bytes(M|N, K) bytes; alpha = 1 is plain
 * MXFP4. */
BLACKHOLE_SM100_API int blackhole_sm100_mxfp4_bf16_gemm(int M, int N, int K, const void* A,
                                                        const void* SFA, const void* B,
                                                        const void* SFB, void* D, float alpha,
                                                        cudaStream_t stream);
/* With an explicit schedule and workspace, as blackhole_sm100_nvfp4_bf16_gemm_ex. */
BLACKHOLE_SM100_API int blackhole_sm100_mxfp4_bf16_gemm_ex(int M, int N, int K, const void* A,
                                                           const void* SFA, const void* B,
                                                           const void* SFB, void* D, float alpha,
                                                           int schedule, void* workspace,
                                                           int64_t workspace_bytes,
                                                           cudaStream_t stream);
/* MXFP8 x MXFP4 -> BF16 (no counterpart in the reference): A (M x K) E4M3, one byte per
 * element, B (N x K) packed E2M1; one UE8M0 scale per 32 elements along K on both, 128x4
 * layout with 32-element groups (blackhole_sm100_mxfp4_sf_storage_bytes bytes each).
 * tcgen05.mma kind::mxf8f6f4.  Shapes and schedules as the MXFP4 calls, plus K % 128 == 0
 * and B 32-byte aligned. */
BLACKHOLE_SM100_API int blackhole_sm100_mxf8f4_bf16_gemm(int M, int N, int K, const void* A,
                                                         const void* SFA, const void* B,
                                                         const void* SFB, void* D, float alpha,
                                                         cudaStream_t stream);
BLACKHOLE_SM100_API int blackhole_sm100_mxf8f4_bf16_gemm_ex(int M, int N, int K, const void* A,
                                                            const void* SFA, const void* B,
                                                            const void* SFB, void* D, float alpha,
                                                            int schedule, void* workspace,
                                                            int64_t workspace_bytes,
                                                            cudaStream_t stream);
/* MXFP8 quantiser (OCP MX v1.0, E4M3 elements, shared exponent floor(log2 amax) - 8, elements
 * rounded to nearest even and saturated at +-448): X rows x K (FP32 when x_is_bf16 == 0, else
 * BF16, K % 32 == 0, 16-byte aligned) -> q (rows*K bytes, 16-byte aligned) and sf (MX layout,
 * padding written 0).  Asynchronous on `stream`. */
BLACKHOLE_SM100_API int blackhole_sm100_mxfp8_quantize(const void* X, int x_is_bf16, int rows,
                                                       int K, void* q, void* sf,
                                                       cudaStream_t stream);

/* Bytes of an (mn, k) MXFP4 scale-factor tensor (rows padded to 128, 32-element groups
 * padded to a multiple of 4); negative on error. */
BLACKHOLE_SM100_API int64_t blackhole_sm100_mxfp4_sf_storage_bytes(int64_t mn, int64_t k);
/* MXFP4 quantiser: X (rows x K, FP32 when x_is_bf16 == 0, else BF16, K % 32 == 0, 16-byte
 * aligned) -> packed E2M1 (rows*K/2 bytes, 16-byte aligned) and UE8M0 scales (padding written
 * 0).  Per 32-block: e = floor(log2(amax_b)) - 2 clamped to [-127, 127], scale 2^e,
 * q = E2M1(x * 2^-e) round-to-nearest-even, saturating at 6. */
BLACKHOLE_SM100_API int blackhole_sm100_mxfp4_quantize(const void* X, int x_is_bf16, int rows,
                                                       int K, void* packed, void* sf,
                                                       cudaStream_t stream);

/* ABI version of the loaded library (BLACKHOLE_SM100_ABI_VERSION). */
BLACKHOLE_SM100_API int blackhole_sm100_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BLACKHOLE_SM100_H */
