/*
 * nvfp4_oracle.h -- CPU restatement of the reference NVFP4 x NVFP4 -> BF16 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or calls this
 * code.  It is the checker for the CUDA path: only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference leg use it.
 *
 * What it restates (reference = Jiaao-Bai/blackhole):
 *   - e2m1 / ue4m3 / bf16 conversions.  The reference delegates these to CUTLASS
 *     (cutlass::float_e2m1_t, cutlass::float_ue4m3_t, cutlass::bfloat16_t), called at
 *     example/nvfp4_bf16_gemm.cu:61-71 and :168.  CUTLASS is an un-vendored submodule of
 *     the reference (.gitmodules:1-3) with no recoverable pinned commit; the semantics
 *     here are pinned against CUTLASS 4.5.0 host code through tests/golden/.
 *   - the 128x4 blocked scale-factor layout, make_layout_SFA/SFB at
 *     include/blackhole/sm120/nvfp4_gemm.hpp:293-298 (CUTLASS Sm1xxBlockScaledConfig),
 *     pinned against the reference header compiled here (tests/golden/).
 *   - the host reference GEMM, example/nvfp4_bf16_gemm.cu:161-168: a sequential FP32
 *     dot product of dequantised values (a*sfa)*(b*sfb), rounded to BF16, extended with
 *     the alpha (global scale) multiply: D = bf16(alpha * acc).
 *   - the BASELINE quantisation recipe (global scale amax/(448*6), per-16 UE4M3 block
 *     scales, E2M1 round-to-nearest-even), which the reference does not ship.
 */
#ifndef BLACKHOLE_NVFP4_ORACLE_H
#define BLACKHOLE_NVFP4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar conversions (CUTLASS 4.5.0 semantics) ---------------------------------- */
uint8_t  bho_e2m1_from_float(float x);     /* RNE, saturate to +-6 (NaN too), sign kept */
float    bho_e2m1_to_float(uint8_t code);  /* low nibble */
uint8_t  bho_ue4m3_from_float(float x);    /* |x|, RNE, saturate to 448, NaN -> 0x7F     */
float    bho_ue4m3_to_float(uint8_t code); /* bit 7 ignored; 0x7F -> NaN                 */
uint16_t bho_bf16_from_float(float x);     /* RNE, NaN -> 0x7FFF                         */
float    bho_bf16_to_float(uint16_t bits);

/* ---- 128x4 blocked scale-factor layout --------------------------------------------- */
/* Byte offset of the scale factor for row `mn`, 16-element K group `kg`, in a tensor
 * whose K extent is `K` elements.  Rows are padded to 128, K groups to multiples of 4. */
int64_t bho_sf_offset(int64_t mn, int64_t kg, int64_t K);
/* Bytes a (MN, K) scale-factor tensor occupies, padding included (the layout's cosize). */
int64_t bho_sf_storage_bytes(int64_t MN, int64_t K);

/* ---- seeded synthetic data --------------------------------------------------------- */
/* out[i] = mean + std * N(0,1) sample number (offset + i) of stream `seed`.
 * splitmix64 counter stream + Box-Muller in double precision. */
void bho_gen_normal(uint64_t seed, int64_t offset, int64_t n, float mean, float std,
                    float* out);
/* Multiply each element by `factor` with probability p (stream `seed`), in place. */
void bho_apply_outliers(uint64_t seed, int64_t n, double p, float factor, float* x);

/* ---- NVFP4 quantiser (BASELINE recipe) --------------------------------------------- */
/* X: rows x K float, K-contiguous, K % 16 == 0.
 * packed: rows*K/2 bytes, low nibble = even k.  sf: bho_sf_storage_bytes(rows, K) bytes,
 * zero-filled first by the caller (padding stays 0).
 * Returns the global scale g = amax/(448*6); alpha for a GEMM is gA*gB. */
float bho_quantize_nvfp4(const float* X, int64_t rows, int64_t K, uint8_t* packed,
                         uint8_t* sf);

/* ---- host reference GEMM ------------------------------------------------------------ */
/* D[m,n] = bf16(alpha * sum_k (a*sfa)*(b*sfb)), sequential FP32 sum in k order.
 * absdot[m*N+n] (optional) = sum_k |a*sfa*b*sfb| (double, for the tolerance).
 * nthreads <= 1 runs single-threaded (the reference loop as-is).                      */
void bho_gemm_ref_full(int64_t M, int64_t N, int64_t K, const uint8_t* A, const uint8_t* SFA,
                       const uint8_t* B, const uint8_t* SFB, float alpha, uint16_t* D,
                       double* absdot, int nthreads);
/* Same arithmetic at S sampled points (ms[i], ns[i]); D_out/absdot have S entries. */
void bho_gemm_ref_sampled(int64_t M, int64_t N, int64_t K, const uint8_t* A,
                          const uint8_t* SFA, const uint8_t* B, const uint8_t* SFB,
                          float alpha, int64_t S, const int64_t* ms, const int64_t* ns,
                          uint16_t* D_out, double* absdot, int nthreads);

/* ---- MXFP4 (OCP MX v1.0: E2M1 elements, one UE8M0 scale per 32 along K) ------------ */
/* Not part of the reference; the sibling format served behind the same operator.  The
 * scale-factor layout is the same 128x4 blocked layout with 32-element K groups (CUTLASS
 * Sm1xxBlockScaledConfig<32>); tests/golden/make_golden_mx.cpp pins it and the decode. */
float   bho_ue8m0_to_float(uint8_t code);  /* 2^(code-127); 0xFF -> NaN */
/* Layout with `vs`-element K groups (vs = 16: NVFP4, vs = 32: MXFP4). */
int64_t bho_sf_offset_vs(int64_t mn, int64_t kg, int64_t K, int vs);
int64_t bho_sf_storage_bytes_vs(int64_t MN, int64_t K, int vs);
/* Per 32-block b: shared exponent e_b = floor(log2(amax_b)) - 2 (2 = emax of E2M1), clamped
 * to [-127, 127] (amax_b subnormal or 0 -> -127); scale code = e_b + 127; element code =
 * e2m1(x * 2^-e_b) (exact scaling, RNE, saturating to 6).  K % 32 == 0; sf zero-filled
 * first by the caller. */
void bho_quantize_mxfp4(const float* X, int64_t rows, int64_t K, uint8_t* packed, uint8_t* sf);
/* Signed E4M3 (OCP E4M3FN): RNE, satfinite to +-448, NaN -> 0x7F; decode (0x7F/0xFF NaN). */
uint8_t bho_e4m3_from_float(float x);
float   bho_e4m3_to_float(uint8_t code);
/* MXFP8 quantiser (E4M3 elements, one UE8M0 scale per 32, shared exponent
 * floor(log2 amax) - 8): q rows*K bytes, sf bho_sf_storage_bytes_vs(rows, K, 32) bytes. */
void bho_quantize_mxfp8(const float* X, int64_t rows, int64_t K, uint8_t* q, uint8_t* sf);
/* The reference GEMM for a format: fmt 0 = NVFP4 (as above), 1 = MXFP4. */
/* fmt: 0 NVFP4 x NVFP4, 1 MXFP4 x MXFP4, 2 MXFP8 A (rows*K bytes) x MXFP4 B. */
void bho_gemm_ref_full_fmt(int fmt, int64_t M, int64_t N, int64_t K, const uint8_t* A,
                           const uint8_t* SFA, const uint8_t* B, const uint8_t* SFB, float alpha,
                           uint16_t* D, double* absdot, int nthreads);
void bho_gemm_ref_sampled_fmt(int fmt, int64_t M, int64_t N, int64_t K, const uint8_t* A,
                              const uint8_t* SFA, const uint8_t* B, const uint8_t* SFB,
                              float alpha, int64_t S, const int64_t* ms, const int64_t* ns,
                              uint16_t* D_out, double* absdot, int nthreads);

/* Tolerance for one element, the one every parity test asserts:
 *   ulp_bf16(max(|ref|,|got|)) + |alpha| * sqrt(K) * 2^-24 * absdot
 * One BF16 ulp of the output (two FP32 sums that differ in their last bits may round to
 * neighbouring BF16 values) plus FP32 reassociation slack.  The products are exact in FP32,
 * so the two sums differ only by rounding: at most K*2^-24*absdot in the worst case, and
 * about sqrt(K)*2^-24 times the size of the partial sums when the rounding errors have
 * random signs, which is what the slack allows (the worst-case form is 169x looser at
 * K = 28672 and lets most elements of a result with a 256-deep k-tile missing through). */
double bho_tolerance(float ref, float got, float alpha, int64_t K, double absdot);
/* The worst-case bound, ulp_bf16 + |alpha| * K * 2^-24 * absdot: the outer limit, reported. */
double bho_tolerance_worst(float ref, float got, float alpha, int64_t K, double absdot);

/* ---- the example's host loop in its own form (example/nvfp4_bf16_gemm.cu:159-168) ---- */
/* Decodes an operand into element values vals[rows*K] and scale values
 * scales[rows*(K/vs)] (fmt_kind 0 NVFP4 vs = 16, 1 MXFP4 vs = 32, 2 MXFP8 vs = 32): the float
 * arrays the example builds before its loop (refA / sfaVal). */
void bho_decode_operand(int fmt_kind, const uint8_t* P, const uint8_t* SF, int64_t rows,
                        int64_t K, float* vals, float* scales);
/* D[m,n] = bf16(alpha * acc), acc += (vA*sA)*(vB*sB) over k in order, every row m of A
 * against every row n of B, rows split over nthreads threads.  Same bits as
 * bho_gemm_ref_full (each product is exact in FP32); this is the loop the CPU baselines time,
 * with the decoding done before it as in the example. */
void bho_ref_loop(int64_t M, int64_t N, int64_t K, int vs, const float* vA, const float* sA,
                  const float* vB, const float* sB, float alpha, uint16_t* D, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
