/*
 * nvfp4_oracle.c — CPU restatement of the reference plugin's NVFP4 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker: the parity tests, the smoke check and
 * the CPU-baseline leg of bench.py call it. The product (my_nvfp4_gemm_b200) never links,
 * loads or falls back to it.
 *
 * It follows, step by step and in the same fp32 operation order:
 *   quantize   : csrc/quantize/quantize_nvfp4.cu:6-35 (kernel), with the conversions of
 *                csrc/common/common.h:65-92 (cvt.rn.satfinite.e2m1x2.f32 / .e4m3x2.f32)
 *   dequantize : csrc/quantize/quantize_nvfp4.cu:44-62, conversions common.h:94-126
 *   GEMM       : csrc/gemm/gemm_nvfp4.cu:147 (block-scaled product, fp32 accumulate) and
 *                :230-231 (epilogue: accumulator / scale, then bf16 round-to-nearest-even)
 *
 * Pinning: the rounding, saturation, signed-zero and NaN encodings below are checked against
 * golden vectors produced by the reference's own quantize/dequant kernels, rebuilt from source
 * for sm_100a and run on a B200 (tests/golden/). The NaN encodings (E2M1_NAN_CODE, BF16_NAN,
 * E4M3_NAN) are hardware conventions of the PTX cvt instructions and are pinned there.
 *
 * Floating point: every step is one IEEE fp32 multiply or divide, rounded to nearest even;
 * build with -ffp-contract=off and without fast-math. Denormals are honoured (the CUDA build
 * of the reference does not flush them); the entry points clear FTZ/DAZ in MXCSR themselves.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <xmmintrin.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define E4M3_NAN 0x7Fu
#define BF16_NAN 0x7FFFu
/* cvt.rn.satfinite.e2m1x2.f32 of a NaN input (E2M1 has no NaN encoding). */
#ifndef E2M1_NAN_CODE
#define E2M1_NAN_CODE 0x7u
#endif

/* ---- MXCSR: make sure no FTZ/DAZ is active while the oracle runs ---------------------- */
static unsigned int ieee_mode_enter(void) {
  unsigned int old = _mm_getcsr();
  _mm_setcsr(old & ~(0x8040u)); /* clear FTZ (bit 15) and DAZ (bit 6) */
  return old;
}
static void ieee_mode_leave(unsigned int old) { _mm_setcsr(old); }

/* ---- scalar conversions ----------------------------------------------------------------- */
static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float nvfp4_oracle_bf16_to_f32(uint16_t h) { return f32_from_bits((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even (cvt.rn.bf16x2.f32 / __float22bfloat162_rn). */
uint16_t nvfp4_oracle_f32_to_bf16(float x) {
  if (isnan(x)) return (uint16_t)BF16_NAN;
  uint32_t u = bits_from_f32(x);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* UE4M3/E4M3 -> fp32 (exact; cvt.rn.f16x2.e4m3x2 then f16 -> f32, common.h:121-126). */
float nvfp4_oracle_e4m3_to_f32(uint8_t v) {
  unsigned s = v >> 7, e = (v >> 3) & 0xFu, m = v & 7u;
  if (e == 0xFu && m == 7u) return s ? -NAN : NAN;
  float r = (e == 0) ? ldexpf((float)m, -9) : ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
  return s ? -r : r;
}

/* fp32 -> E4M3, round to nearest even with saturation to +-448 (cvt.rn.satfinite.e4m3x2.f32,
 * common.h:85-92). NaN -> 0x7F. */
uint8_t nvfp4_oracle_f32_to_e4m3(float x) {
  if (isnan(x)) return (uint8_t)E4M3_NAN;
  uint8_t sign = signbit(x) ? 0x80u : 0u;
  float a = fabsf(x);
  if (a >= 448.0f) return sign | 0x7Eu;
  if (a == 0.0f) return sign;
  int e;
  (void)frexpf(a, &e);              /* a = f * 2^e, f in [0.5, 1) */
  int ex = e - 1;                   /* floor(log2(a)) */
  if (ex < -6) ex = -6;             /* subnormal range shares the 2^-9 quantum */
  float q = ldexpf(1.0f, ex - 3);   /* spacing of E4M3 values around a */
  float r = nearbyintf(a / q) * q;  /* a / q is exact (power-of-two q); RNE */
  if (r == 0.0f) return sign;
  (void)frexpf(r, &e);
  int E = e - 1;
  if (E < -6) return sign | (uint8_t)(r / ldexpf(1.0f, -9));            /* subnormal */
  unsigned m = (unsigned)((r / ldexpf(1.0f, E) - 1.0f) * 8.0f);
  return sign | (uint8_t)(((unsigned)(E + 7) << 3) | m);
}

/* E2M1 code (low 4 bits) -> fp32. */
float nvfp4_oracle_e2m1_to_f32(uint8_t code) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float r = mag[code & 7u];
  return (code & 8u) ? -r : r;
}

/* fp32 -> E2M1 code, round to nearest even, saturating at +-6 (cvt.rn.satfinite.e2m1x2.f32,
 * common.h:65-83). The sign bit is kept, so -0 and small negatives give 0x8. */
uint8_t nvfp4_oracle_f32_to_e2m1(float x) {
  if (isnan(x)) return (uint8_t)E2M1_NAN_CODE;
  uint8_t sign = signbit(x) ? 8u : 0u;
  float a = fabsf(x);
  uint8_t c;
  if (a <= 0.25f) c = 0;        /* tie 0.25 -> 0 (even)   */
  else if (a < 0.75f) c = 1;    /* 0.5                    */
  else if (a <= 1.25f) c = 2;   /* tie 0.75 -> 1.0, tie 1.25 -> 1.0 */
  else if (a < 1.75f) c = 3;    /* 1.5                    */
  else if (a <= 2.5f) c = 4;    /* tie 1.75 -> 2, tie 2.5 -> 2 */
  else if (a < 3.5f) c = 5;     /* 3                      */
  else if (a <= 5.0f) c = 6;    /* tie 3.5 -> 4, tie 5 -> 4 */
  else c = 7;                   /* 6, saturating (inf included) */
  return sign | c;
}

/* ---- one 16-element block (quantize_nvfp4.cu:6-35) -------------------------------------- */
static void quantize_block(const uint16_t* xb, float s, float rcp_s, uint8_t* qb, uint8_t* sfb) {
  /* amax = NaN-propagating max of |x_i| seeded with the bf16 bit pattern 0x0001 (:14-23).
   * For non-NaN bf16 magnitudes the bit pattern orders like the value. */
  uint16_t amax = 0x0001u;
  int any_nan = 0;
  for (int i = 0; i < 16; ++i) {
    uint16_t a = (uint16_t)(xb[i] & 0x7FFFu);
    if (a > 0x7F80u) any_nan = 1;
    else if (a > amax) amax = a;
  }
  float famax = any_nan ? NAN : nvfp4_oracle_bf16_to_f32(amax);
  const float rcp6 = 1.0f / 6.0f;           /* the fp32 constant 0.16666667f (:11-12) */
  volatile float t = famax * s;             /* (amax * s) first ... (:24) */
  float tt = t * rcp6;                      /* ... then * (1/6) */
  uint8_t sf = nvfp4_oracle_f32_to_e4m3(tt);
  *sfb = sf;
  volatile float den = nvfp4_oracle_e4m3_to_f32(sf) * rcp_s;
  float os = 1.0f / den;                    /* __frcp_rn(f32(sf) * __frcp_rn(s)) (:27) */
  for (int j = 0; j < 8; ++j) {
    float y0 = nvfp4_oracle_bf16_to_f32(xb[2 * j]) * os;
    float y1 = nvfp4_oracle_bf16_to_f32(xb[2 * j + 1]) * os;
    qb[j] = (uint8_t)(nvfp4_oracle_f32_to_e2m1(y0) | (nvfp4_oracle_f32_to_e2m1(y1) << 4));
  }
}

/* Quantize a flat bf16 array of `numel` elements (numel % 16 == 0). */
void nvfp4_oracle_quantize(const uint16_t* x, float s, int64_t numel, uint8_t* q, uint8_t* sf) {
  const int64_t nblk = numel / 16;
  const float rcp_s = 1.0f / s;
#pragma omp parallel
  {
    unsigned int mode = ieee_mode_enter();
#pragma omp for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) quantize_block(x + b * 16, s, rcp_s, q + b * 8, sf + b);
    ieee_mode_leave(mode);
  }
}

/* Dequantize `n_bytes` packed bytes (n_bytes % 8 == 0) -> 2*n_bytes bf16 (:44-62). */
void nvfp4_oracle_dequantize(const uint8_t* q, float s, const uint8_t* sf, int64_t n_bytes,
                             uint16_t* y) {
  const int64_t nblk = n_bytes / 8;
#pragma omp parallel
  {
    unsigned int mode = ieee_mode_enter();
    const float rcp_s = 1.0f / s;
#pragma omp for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) {
      float scale = nvfp4_oracle_e4m3_to_f32(sf[b]) * rcp_s;   /* (:49) */
      for (int j = 0; j < 8; ++j) {
        uint8_t byte = q[b * 8 + j];
        y[b * 16 + 2 * j] = nvfp4_oracle_f32_to_bf16(nvfp4_oracle_e2m1_to_f32(byte & 0xFu) * scale);
        y[b * 16 + 2 * j + 1] = nvfp4_oracle_f32_to_bf16(nvfp4_oracle_e2m1_to_f32(byte >> 4) * scale);
      }
    }
    ieee_mode_leave(mode);
  }
}

/* Decode a packed [rows, k] operand to fp32 values e2m1 * f32(sf) WITHOUT the global scale,
 * which is what the block-scaled MMA multiplies (gemm_nvfp4.cu:147). Exact in fp32. */
void nvfp4_oracle_decode_scaled(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t k,
                                float* out) {
  const int64_t nblk = rows * (k / 16);
#pragma omp parallel
  {
    unsigned int mode = ieee_mode_enter();
#pragma omp for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) {
      float sc = nvfp4_oracle_e4m3_to_f32(sf[b]);
      for (int j = 0; j < 8; ++j) {
        uint8_t byte = q[b * 8 + j];
        out[b * 16 + 2 * j] = nvfp4_oracle_e2m1_to_f32(byte & 0xFu) * sc;
        out[b * 16 + 2 * j + 1] = nvfp4_oracle_e2m1_to_f32(byte >> 4) * sc;
      }
    }
    ieee_mode_leave(mode);
  }
}

/* Epilogue of the reference GEMM (gemm_nvfp4.cu:230-231): fp32 accumulator / scale -> bf16. */
uint16_t nvfp4_oracle_epilogue(float acc, float scale) {
  volatile float d = acc / scale;
  return nvfp4_oracle_f32_to_bf16(d);
}

/* Reference GEMM on decoded operands: D[m,n] = bf16( fp32(sum_k fa[m,k] fb[n,k]) / scale ).
 * The sum is taken in double (the tensor core's fp32 summation order is unspecified), rounded
 * once to fp32, then divided as in the reference epilogue. d_f32 (optional) receives the
 * unrounded fp32 quotient. */
void nvfp4_oracle_gemm(const uint8_t* A, const uint8_t* B, const uint8_t* A_sf,
                       const uint8_t* B_sf, float scale, int64_t M, int64_t N, int64_t K,
                       float* fa_scratch, float* fb_scratch, float* d_f32, uint16_t* d_bf16) {
  nvfp4_oracle_decode_scaled(A, A_sf, M, K, fa_scratch);
  nvfp4_oracle_decode_scaled(B, B_sf, N, K, fb_scratch);
#pragma omp parallel
  {
    unsigned int mode = ieee_mode_enter();
#pragma omp for schedule(static) collapse(2)
    for (int64_t m = 0; m < M; ++m) {
      for (int64_t n = 0; n < N; ++n) {
        const float* a = fa_scratch + m * K;
        const float* b = fb_scratch + n * K;
        double acc = 0.0;
        for (int64_t k = 0; k < K; ++k) acc += (double)a[k] * (double)b[k];
        volatile float accf = (float)acc;
        volatile float d = accf / scale;
        if (d_f32) d_f32[m * N + n] = d;
        if (d_bf16) d_bf16[m * N + n] = nvfp4_oracle_f32_to_bf16(d);
      }
    }
    ieee_mode_leave(mode);
  }
}

/* Threads the OpenMP runtime will use (reported by the CPU baseline). */
int nvfp4_oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
