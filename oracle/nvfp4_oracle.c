/*
 * nvfp4_oracle.c -- CPU restatement of the reference NVFP4 GEMM path (see the header).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the product.
 * Built with -ffp-contract=off so that `acc + a*b` is a separate multiply and add,
 * exactly like the reference loop compiled for x86-64 (example/nvfp4_bf16_gemm.cu:161-166).
 */
#include "nvfp4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------ */
/* Conversions.  Each one restates the published rounding rule (IEEE round to nearest,  */
/* ties to even) for the target format and the saturation / NaN conventions that        */
/* CUTLASS 4.5.0's host converters use; tests/golden pins every branch.                  */
/* ------------------------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* E2M1 magnitudes by code: 0, 0.5, 1, 1.5, 2, 3, 4, 6.  A midpoint rounds to the code
 * whose last bit is 0 (the even one).  Used by cutlass::float_e2m1_t(float), called at
 * example/nvfp4_bf16_gemm.cu:61-64. */
uint8_t bho_e2m1_from_float(float x) {
  uint32_t u = f2u(x);
  uint8_t sign = (uint8_t)((u >> 31) << 3);
  if (isnan(x)) return (uint8_t)(sign | 0x7); /* CUTLASS saturates NaN to +-6 by its sign */
  float a = fabsf(x);
  uint8_t mag;
  if (a <= 0.25f)      mag = 0;          /* tie 0.25 -> 0.0 (code 0, even)  */
  else if (a < 0.75f)  mag = 1;          /* tie 0.75 -> 1.0 (code 2, even)  */
  else if (a <= 1.25f) mag = 2;          /* tie 1.25 -> 1.0 (code 2)        */
  else if (a < 1.75f)  mag = 3;          /* tie 1.75 -> 2.0 (code 4)        */
  else if (a <= 2.5f)  mag = 4;          /* tie 2.5  -> 2.0 (code 4)        */
  else if (a < 3.5f)   mag = 5;          /* tie 3.5  -> 4.0 (code 6)        */
  else if (a <= 5.0f)  mag = 6;          /* tie 5.0  -> 4.0 (code 6)        */
  else                 mag = 7;          /* everything above saturates to 6 */
  return (uint8_t)(sign | mag);
}

float bho_e2m1_to_float(uint8_t code) {
  static const float mags[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float v = mags[code & 7];
  return (code & 8) ? -v : v;
}

/* Unsigned E4M3 (bias 7, 3 mantissa bits, subnormal step 2^-9, max 448, 0x7F = NaN).
 * The sign of the input is dropped (|x|).  Used by cutlass::float_ue4m3_t(float),
 * example/nvfp4_bf16_gemm.cu:66-70. */
uint8_t bho_ue4m3_from_float(float x) {
  if (isnan(x)) return 0x7F;
  double a = fabs((double)x);
  if (a >= 448.0) return 0x7E;           /* saturate (inf included) */
  if (a < 0.015625) {                    /* below the smallest normal 2^-6 */
    double m = nearbyint(a * 512.0);     /* exact scaling; ties to even */
    return (uint8_t)m;                   /* m == 8 is code 0x08 = 2^-6: consistent */
  }
  int e;
  double fr = frexp(a, &e);              /* a = fr * 2^e, fr in [0.5, 1) */
  e -= 1;                                /* a = (2*fr) * 2^e, 2*fr in [1, 2) */
  double m = nearbyint((2.0 * fr - 1.0) * 8.0);
  if (m >= 8.0) { m = 0.0; e += 1; }
  int code = ((e + 7) << 3) | (int)m;
  if (code >= 0x7F) code = 0x7E;
  return (uint8_t)code;
}

float bho_ue4m3_to_float(uint8_t code) {
  code &= 0x7F;
  if (code == 0x7F) return NAN;
  int e = code >> 3, m = code & 7;
  if (e == 0) return (float)ldexp((double)m, -9);
  return (float)ldexp(1.0 + m / 8.0, e - 7);
}

uint16_t bho_bf16_from_float(float x) {
  if (isnan(x)) return 0x7FFF;
  uint32_t u = f2u(x);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float bho_bf16_to_float(uint16_t bits) { return u2f((uint32_t)bits << 16); }

/* ------------------------------------------------------------------------------------ */
/* 128x4 blocked scale-factor layout (CUTLASS Sm1xxBlockScaledConfig, reached through    */
/* make_layout_SFA/SFB, include/blackhole/sm120/nvfp4_gemm.hpp:293-298).                 */
/* A 512-byte atom holds 128 rows x 4 K-groups: byte (mn%32)*16 + ((mn/32)%4)*4 + kg%4.   */
/* Atoms advance along K first, then along MN.                                           */
/* ------------------------------------------------------------------------------------ */
int64_t bho_sf_offset(int64_t mn, int64_t kg, int64_t K) {
  int64_t kg_blocks = (K / 16 + 3) / 4;
  return ((mn / 128) * kg_blocks + kg / 4) * 512 + (mn % 32) * 16 + ((mn / 32) % 4) * 4 +
         (kg % 4);
}

int64_t bho_sf_storage_bytes(int64_t MN, int64_t K) {
  int64_t kg_blocks = (K / 16 + 3) / 4;
  return ((MN + 127) / 128) * kg_blocks * 512;
}

/* The same atom with vs-element K groups (MXFP4: vs = 32). */
int64_t bho_sf_offset_vs(int64_t mn, int64_t kg, int64_t K, int vs) {
  int64_t kg_blocks = (K / vs + 3) / 4;
  return ((mn / 128) * kg_blocks + kg / 4) * 512 + (mn % 32) * 16 + ((mn / 32) % 4) * 4 +
         (kg % 4);
}

int64_t bho_sf_storage_bytes_vs(int64_t MN, int64_t K, int vs) {
  return ((MN + 127) / 128) * ((K / vs + 3) / 4) * 512;
}

/* Signed E4M3 (OCP E4M3FN: bias 7, 3 mantissa bits, subnormal step 2^-9, max 448, no
 * infinities, 0x7F / 0xFF NaN): round to nearest even on |x| as for UE4M3, finite values
 * past 448 and infinities saturate to +-448, NaN becomes 0x7F (sign dropped), the sign of
 * zero and of values that round to zero is kept.  The conventions of
 * cutlass::float_e4m3_t(float) in CUTLASS 4.5.0 and of the satfinite e4m3 conversion. */
uint8_t bho_e4m3_from_float(float x) {
  if (isnan(x)) return 0x7F;
  uint8_t sign = (uint8_t)((f2u(x) >> 31) << 7);
  return (uint8_t)(sign | bho_ue4m3_from_float(x));
}

float bho_e4m3_to_float(uint8_t code) {
  float v = bho_ue4m3_to_float((uint8_t)(code & 0x7F));
  return (code & 0x80) ? -v : v;
}

/* UE8M0: an 8-bit biased exponent, value 2^(code - 127); code 0xFF is NaN. */
float bho_ue8m0_to_float(uint8_t code) {
  if (code == 0xFF) return NAN;
  return (float)ldexp(1.0, (int)code - 127);
}

/* ------------------------------------------------------------------------------------ */
/* Seeded normal generator: splitmix64 over a counter, Box-Muller in double.             */
/* ------------------------------------------------------------------------------------ */
static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t rand_at(uint64_t seed, uint64_t i) {
  return mix64(seed * 0xD1B54A32D192ED03ull + (i + 1) * 0x9E3779B97F4A7C15ull);
}

void bho_gen_normal(uint64_t seed, int64_t offset, int64_t n, float mean, float std,
                    float* out) {
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t j = 0; j < n; ++j) {
    int64_t i = offset + j;
    int64_t pair = i >> 1;
    double u1 = ((double)(rand_at(seed, 2 * (uint64_t)pair) >> 11) + 1.0) * 0x1.0p-53;
    double u2 = (double)(rand_at(seed, 2 * (uint64_t)pair + 1) >> 11) * 0x1.0p-53;
    double r = sqrt(-2.0 * log(u1));
    double z = (i & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
    out[j] = (float)(mean + std * z);
  }
}

void bho_apply_outliers(uint64_t seed, int64_t n, double p, float factor, float* x) {
  uint64_t thresh = (uint64_t)(p * 18446744073709551616.0);
  for (int64_t i = 0; i < n; ++i)
    if (rand_at(seed ^ 0x5bd1e9955bd1e995ull, (uint64_t)i) < thresh) x[i] *= factor;
}

/* ------------------------------------------------------------------------------------ */
/* Quantiser: g = amax/(448*6); s_b = ue4m3((amax_b/6)/g); q = e2m1(x/(s_b*g)).           */
/* Every step is one IEEE float operation, so a device quantiser doing the same ops in    */
/* the same order reproduces it bit for bit.                                              */
/* ------------------------------------------------------------------------------------ */
float bho_quantize_nvfp4(const float* X, int64_t rows, int64_t K, uint8_t* packed,
                         uint8_t* sf) {
  float amax = 0.0f;
  for (int64_t i = 0; i < rows * K; ++i) {
    float a = fabsf(X[i]);
    if (a > amax) amax = a;
  }
  float g = amax / 2688.0f;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < K / 16; ++b) {
      const float* x = X + r * K + b * 16;
      float amax_b = 0.0f;
      for (int i = 0; i < 16; ++i) {
        float a = fabsf(x[i]);
        if (a > amax_b) amax_b = a;
      }
      uint8_t s_code = 0;
      float s_val = 0.0f;
      if (g > 0.0f) {
        s_code = bho_ue4m3_from_float((amax_b / 6.0f) / g);
        s_val = bho_ue4m3_to_float(s_code);
      }
      sf[bho_sf_offset(r, b, K)] = s_code;
      float scale = s_val * g;
      uint8_t* dst = packed + (r * K + b * 16) / 2;
      for (int i = 0; i < 16; i += 2) {
        uint8_t lo = 0, hi = 0;
        if (s_val != 0.0f) {
          lo = bho_e2m1_from_float(x[i] / scale);
          hi = bho_e2m1_from_float(x[i + 1] / scale);
        }
        dst[i / 2] = (uint8_t)(lo | (hi << 4));
      }
    }
  }
  return g;
}

/* ------------------------------------------------------------------------------------ */
/* MXFP4 quantiser (OCP Microscaling Formats v1.0, E2M1 elements, X = 2^(floor(log2 amax) */
/* - emax_elem)).  The exponent is read from the float's bits and the element scaling is   */
/* a multiplication by an exact power of two, so a device quantiser reproduces it exactly. */
/* ------------------------------------------------------------------------------------ */
void bho_quantize_mxfp4(const float* X, int64_t rows, int64_t K, uint8_t* packed, uint8_t* sf) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < K / 32; ++b) {
      const float* x = X + r * K + b * 32;
      float amax_b = 0.0f;
      for (int i = 0; i < 32; ++i) {
        float a = fabsf(x[i]);
        if (a > amax_b) amax_b = a;
      }
      int ebits = (int)((f2u(amax_b) >> 23) & 0xFF); /* 0 for zero and subnormals */
      int e = ebits == 0 ? -127 : (ebits - 127) - 2;
      if (e < -127) e = -127;
      if (e > 127) e = 127;
      sf[bho_sf_offset_vs(r, b, K, 32)] = (uint8_t)(e + 127);
      const float inv = u2f((uint32_t)(127 - e) << 23); /* 2^-e, a normal float for e <= 126 */
      uint8_t* dst = packed + (r * K + b * 32) / 2;
      for (int i = 0; i < 32; i += 2) {
        uint8_t lo = bho_e2m1_from_float(x[i] * inv);
        uint8_t hi = bho_e2m1_from_float(x[i + 1] * inv);
        dst[i / 2] = (uint8_t)(lo | (hi << 4));
      }
    }
  }
}

/* MXFP8 (E4M3 elements) with the same rule: emax_elem = 8 (448 = 1.75 * 2^8), so the
 * shared exponent is floor(log2 amax) - 8 and scaled elements stay below 2^9; those past
 * 448 saturate. */
void bho_quantize_mxfp8(const float* X, int64_t rows, int64_t K, uint8_t* q, uint8_t* sf) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < K / 32; ++b) {
      const float* x = X + r * K + b * 32;
      float amax_b = 0.0f;
      for (int i = 0; i < 32; ++i) {
        float a = fabsf(x[i]);
        if (a > amax_b) amax_b = a;
      }
      int ebits = (int)((f2u(amax_b) >> 23) & 0xFF);
      int e = ebits == 0 ? -127 : (ebits - 127) - 8;
      if (e < -127) e = -127;
      if (e > 127) e = 127;
      sf[bho_sf_offset_vs(r, b, K, 32)] = (uint8_t)(e + 127);
      const float inv = u2f((uint32_t)(127 - e) << 23);
      for (int i = 0; i < 32; ++i) q[r * K + b * 32 + i] = bho_e4m3_from_float(x[i] * inv);
    }
  }
}

/* ------------------------------------------------------------------------------------ */
/* Host reference GEMM (example/nvfp4_bf16_gemm.cu:161-168, plus alpha).                  */
/* Formats: 0 NVFP4 x NVFP4, 1 MXFP4 x MXFP4, 2 MXFP8 (A, one byte per element) x MXFP4.  */
/* ------------------------------------------------------------------------------------ */
/* Operand element kinds: 0 NVFP4, 1 MXFP4, 2 MXFP8. */
static int a_kind(int fmt) { return fmt; }
static int b_kind(int fmt) { return fmt == 2 ? 1 : fmt; }

static void dequant_row_fmt(int fmt, const uint8_t* P, const uint8_t* SF, int64_t row,
                            int64_t K, float* out) {
  if (fmt == 2) {
    const uint8_t* p = P + row * K;
    for (int64_t k = 0; k < K; ++k)
      out[k] = bho_e4m3_to_float(p[k]) * bho_ue8m0_to_float(SF[bho_sf_offset_vs(row, k / 32, K, 32)]);
    return;
  }
  const uint8_t* p = P + row * (K / 2);
  for (int64_t k = 0; k < K; k += 2) {
    uint8_t byte = p[k / 2];
    float s = fmt == 1 ? bho_ue8m0_to_float(SF[bho_sf_offset_vs(row, k / 32, K, 32)])
                       : bho_ue4m3_to_float(SF[bho_sf_offset(row, k / 16, K)]);
    out[k] = bho_e2m1_to_float(byte & 0xF) * s;
    out[k + 1] = bho_e2m1_to_float(byte >> 4) * s;
  }
}
static void dequant_row(const uint8_t* P, const uint8_t* SF, int64_t row, int64_t K,
                        float* out) {
  dequant_row_fmt(0, P, SF, row, K, out);
}

static float dot_seq(const float* a, const float* b, int64_t K, double* absdot) {
  float acc = 0.0f;
  double s = 0.0;
  for (int64_t k = 0; k < K; ++k) {
    float p = a[k] * b[k];
    acc = acc + p;
    s += fabs((double)p);
  }
  if (absdot) *absdot = s;
  return acc;
}

typedef struct {
  int64_t M, N, K;
  const uint8_t *A, *SFA, *B, *SFB;
  float alpha;
  uint16_t* D;
  double* absdot;
  const float* Bdq; /* N x K dequantised B */
  int64_t m0, m1;
  /* sampled mode */
  int64_t S;
  const int64_t *ms, *ns;
  int sampled;
  int fmt;
} gemm_job;

static void* gemm_worker(void* arg) {
  gemm_job* j = (gemm_job*)arg;
  float* arow = (float*)malloc(sizeof(float) * (size_t)j->K);
  if (!j->sampled) {
    for (int64_t m = j->m0; m < j->m1; ++m) {
      dequant_row_fmt(a_kind(j->fmt), j->A, j->SFA, m, j->K, arow);
      for (int64_t n = 0; n < j->N; ++n) {
        double ad;
        float acc = dot_seq(arow, j->Bdq + n * j->K, j->K, &ad);
        j->D[m * j->N + n] = bho_bf16_from_float(j->alpha * acc);
        if (j->absdot) j->absdot[m * j->N + n] = ad;
      }
    }
  } else {
    float* brow = (float*)malloc(sizeof(float) * (size_t)j->K);
    for (int64_t s = j->m0; s < j->m1; ++s) {
      dequant_row_fmt(a_kind(j->fmt), j->A, j->SFA, j->ms[s], j->K, arow);
      dequant_row_fmt(b_kind(j->fmt), j->B, j->SFB, j->ns[s], j->K, brow);
      double ad;
      float acc = dot_seq(arow, brow, j->K, &ad);
      j->D[s] = bho_bf16_from_float(j->alpha * acc);
      if (j->absdot) j->absdot[s] = ad;
    }
    free(brow);
  }
  free(arow);
  return NULL;
}

static void run_jobs(gemm_job* base, int64_t total, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > total) nthreads = (int)(total > 0 ? total : 1);
  pthread_t tid[256];
  gemm_job jobs[256];
  for (int t = 0; t < nthreads; ++t) {
    jobs[t] = *base;
    jobs[t].m0 = total * t / nthreads;
    jobs[t].m1 = total * (t + 1) / nthreads;
  }
  if (nthreads == 1) {
    gemm_worker(&jobs[0]);
    return;
  }
  for (int t = 0; t < nthreads; ++t) pthread_create(&tid[t], NULL, gemm_worker, &jobs[t]);
  for (int t = 0; t < nthreads; ++t) pthread_join(tid[t], NULL);
}

typedef struct {
  const uint8_t *P, *SF;
  int64_t K, r0, r1;
  float* out;
  int fmt;
} dequant_job;

static void* dequant_worker(void* arg) {
  dequant_job* j = (dequant_job*)arg;
  for (int64_t r = j->r0; r < j->r1; ++r)
    dequant_row_fmt(j->fmt, j->P, j->SF, r, j->K, j->out + r * j->K);
  return NULL;
}

static void dequant_rows_parallel(int fmt, const uint8_t* P, const uint8_t* SF, int64_t rows,
                                  int64_t K, float* out, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > rows) nthreads = (int)(rows > 0 ? rows : 1);
  pthread_t tid[256];
  dequant_job jobs[256];
  for (int t = 0; t < nthreads; ++t) {
    dequant_job j = {P, SF, K, rows * t / nthreads, rows * (t + 1) / nthreads, out, fmt};
    jobs[t] = j;
  }
  if (nthreads == 1) {
    dequant_worker(&jobs[0]);
    return;
  }
  for (int t = 0; t < nthreads; ++t) pthread_create(&tid[t], NULL, dequant_worker, &jobs[t]);
  for (int t = 0; t < nthreads; ++t) pthread_join(tid[t], NULL);
}

void bho_gemm_ref_full_fmt(int fmt, int64_t M, int64_t N, int64_t K, const uint8_t* A,
                           const uint8_t* SFA, const uint8_t* B, const uint8_t* SFB, float alpha,
                           uint16_t* D, double* absdot, int nthreads) {
  float* Bdq = (float*)malloc(sizeof(float) * (size_t)(N * K));
  dequant_rows_parallel(b_kind(fmt), B, SFB, N, K, Bdq, nthreads);
  gemm_job job = {M, N, K, A, SFA, B, SFB, alpha, D, absdot, Bdq, 0, 0, 0, NULL, NULL, 0, fmt};
  run_jobs(&job, M, nthreads);
  free(Bdq);
}

void bho_gemm_ref_sampled_fmt(int fmt, int64_t M, int64_t N, int64_t K, const uint8_t* A,
                              const uint8_t* SFA, const uint8_t* B, const uint8_t* SFB,
                              float alpha, int64_t S, const int64_t* ms, const int64_t* ns,
                              uint16_t* D_out, double* absdot, int nthreads) {
  gemm_job job = {M, N, K, A, SFA, B, SFB, alpha, D_out, absdot, NULL, 0, 0, S, ms, ns, 1, fmt};
  run_jobs(&job, S, nthreads);
}

void bho_gemm_ref_full(int64_t M, int64_t N, int64_t K, const uint8_t* A, const uint8_t* SFA,
                       const uint8_t* B, const uint8_t* SFB, float alpha, uint16_t* D,
                       double* absdot, int nthreads) {
  bho_gemm_ref_full_fmt(0, M, N, K, A, SFA, B, SFB, alpha, D, absdot, nthreads);
}

void bho_gemm_ref_sampled(int64_t M, int64_t N, int64_t K, const uint8_t* A,
                          const uint8_t* SFA, const uint8_t* B, const uint8_t* SFB,
                          float alpha, int64_t S, const int64_t* ms, const int64_t* ns,
                          uint16_t* D_out, double* absdot, int nthreads) {
  bho_gemm_ref_sampled_fmt(0, M, N, K, A, SFA, B, SFB, alpha, S, ms, ns, D_out, absdot,
                           nthreads);
}

static double bf16_ulp_of(float ref, float got) {
  float a = fabsf(ref) > fabsf(got) ? fabsf(ref) : fabsf(got);
  if (!(a >= 1.1754943508222875e-38f)) a = 1.1754943508222875e-38f;
  int e;
  frexp((double)a, &e);                  /* a in [2^(e-1), 2^e) */
  return ldexp(1.0, (e - 1) - 7);        /* bf16 keeps 7 fraction bits */
}

double bho_tolerance(float ref, float got, float alpha, int64_t K, double absdot) {
  return bf16_ulp_of(ref, got) + fabs((double)alpha) * sqrt((double)K) * 0x1.0p-24 * absdot;
}

double bho_tolerance_worst(float ref, float got, float alpha, int64_t K, double absdot) {
  return bf16_ulp_of(ref, got) + fabs((double)alpha) * (double)K * 0x1.0p-24 * absdot;
}

/* ------------------------------------------------------------------------------------ */
/* The example's host loop in its own form (example/nvfp4_bf16_gemm.cu:159-168): element  */
/* values and per-group scale values as float arrays built before the loop, and inside it */
/* a = vA*sA, b = vB*sB, acc += a*b in k order.                                            */
/* ------------------------------------------------------------------------------------ */
void bho_decode_operand(int fmt_kind, const uint8_t* P, const uint8_t* SF, int64_t rows,
                        int64_t K, float* vals, float* scales) {
  const int vs = fmt_kind == 0 ? 16 : 32;
  const int64_t kg = K / vs;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g = 0; g < kg; ++g)
      scales[r * kg + g] = fmt_kind == 0 ? bho_ue4m3_to_float(SF[bho_sf_offset(r, g, K)])
                                         : bho_ue8m0_to_float(SF[bho_sf_offset_vs(r, g, K, 32)]);
    if (fmt_kind == 2) {
      for (int64_t k = 0; k < K; ++k) vals[r * K + k] = bho_e4m3_to_float(P[r * K + k]);
    } else {
      const uint8_t* p = P + r * (K / 2);
      for (int64_t k = 0; k < K; k += 2) {
        vals[r * K + k] = bho_e2m1_to_float(p[k / 2] & 0xF);
        vals[r * K + k + 1] = bho_e2m1_to_float(p[k / 2] >> 4);
      }
    }
  }
}

typedef struct {
  int64_t N, K, vs, m0, m1;
  const float *vA, *sA, *vB, *sB;
  float alpha;
  uint16_t* D;
} loop_job;

/* One output row against every row of B; VS is a compile-time constant as in the example
 * (k / KT::SFVecSize), so the group index is a shift, not a division. */
#define BHO_LOOP_ROWS(VS)                                                         \
  for (int64_t m = j->m0; m < j->m1; ++m) {                                       \
    const float* va = j->vA + m * K;                                              \
    const float* sa = j->sA + m * (K / (VS));                                     \
    for (int64_t n = 0; n < j->N; ++n) {                                          \
      const float* vb = j->vB + n * K;                                            \
      const float* sb = j->sB + n * (K / (VS));                                   \
      float acc = 0.f;                                                            \
      for (int64_t k = 0; k < K; ++k) {                                           \
        float a = va[k] * sa[k / (VS)];                                           \
        float b = vb[k] * sb[k / (VS)];                                           \
        acc += a * b;                                                             \
      }                                                                           \
      j->D[m * j->N + n] = bho_bf16_from_float(j->alpha * acc);                   \
    }                                                                             \
  }

static void* loop_worker(void* arg) {
  loop_job* j = (loop_job*)arg;
  const int64_t K = j->K;
  if (j->vs == 16) {
    BHO_LOOP_ROWS(16)
  } else {
    BHO_LOOP_ROWS(32)
  }
  return NULL;
}

void bho_ref_loop(int64_t M, int64_t N, int64_t K, int vs, const float* vA, const float* sA,
                  const float* vB, const float* sB, float alpha, uint16_t* D, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > M) nthreads = (int)(M > 0 ? M : 1);
  pthread_t tid[256];
  loop_job jobs[256];
  for (int t = 0; t < nthreads; ++t) {
    loop_job j = {N, K, vs, M * t / nthreads, M * (t + 1) / nthreads, vA, sA, vB, sB, alpha, D};
    jobs[t] = j;
  }
  if (nthreads == 1) {
    loop_worker(&jobs[0]);
    return;
  }
  for (int t = 0; t < nthreads; ++t) pthread_create(&tid[t], NULL, loop_worker, &jobs[t]);
  for (int t = 0; t < nthreads; ++t) pthread_join(tid[t], NULL);
}
