/*
 * ody_oracle.c -- CPU restatement of Odyssey's mixed-precision update path.
 *
 * TEST INFRASTRUCTURE ONLY (see ody_oracle.h).  Build: oracle/Makefile
 * (gcc -O3 -ffp-contract=off -fno-fast-math -fopenmp); no FMA contraction
 * and no flush-to-zero, so every float operation below is one IEEE-rounded
 * operation, as in the reference's tensor-at-a-time Mojo code.
 *
 * Citations are file:line inside HomericIntelligence/Odyssey.
 */
#include "ody_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;
void ora_set_threads(int n) { g_threads = n; }
int ora_get_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}
#define ORA_NT ora_get_threads()

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------------------ */
/* Generic IEEE round-to-nearest-even of a finite, non-negative float32     */
/* (given as its bit pattern) into a binary format with `mbits` mantissa    */
/* bits, exponent bias `bias` and minimum normal exponent `emin`.  Returns  */
/* the magnitude code (exponent << mbits | mantissa) with no overflow       */
/* handling; callers clamp.  This is the cast the Mojo stdlib performs for  */
/* Float32 -> Float16/BFloat16/float8 (any_tensor.mojo:1343-1366,           */
/* tensor_dtype_conv.mojo:54-57, nvfp4.mojo:80-81), assumed RNE.            */
/* ------------------------------------------------------------------------ */
static uint32_t rne_code(uint32_t a, int mbits, int bias, int emin) {
  int e32 = (int)(a >> 23);
  uint32_t m24;
  int E;
  if (e32 == 0) { /* float32 subnormal */
    m24 = a & 0x7fffff;
    E = -126;
  } else {
    m24 = (a & 0x7fffff) | 0x800000;
    E = e32 - 127;
  }
  if (m24 == 0) return 0;
  int shift;
  uint32_t base;
  if (E >= emin) {
    shift = 23 - mbits;
    base = ((uint32_t)(E + bias) << mbits) - (1u << mbits);
  } else {
    shift = 23 - mbits + (emin - E);
    base = 0;
  }
  uint32_t q;
  if (shift >= 32) {
    q = 0;
  } else if (shift == 0) {
    q = m24;
  } else {
    uint32_t rem = m24 & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    q = m24 >> shift;
    if (rem > half || (rem == half && (q & 1u))) q++;
  }
  return base + q;
}

uint16_t ora_f32_to_f16(float x) {
  uint32_t u = f2u(x);
  uint16_t s = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(s | 0x7fffu);
  if (a == 0x7f800000u) return (uint16_t)(s | 0x7c00u);
  uint32_t c = rne_code(a, 10, 15, -14);
  if (c >= 0x7c00u) c = 0x7c00u;
  return (uint16_t)(s | c);
}

float ora_f16_to_f32(uint16_t h) {
  uint32_t s = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
  float v;
  if (e == 0)
    v = ldexpf((float)m, -24);
  else if (e == 31)
    return u2f(s | 0x7f800000u | (m << 13));
  else
    v = ldexpf((float)(m | 0x400u), (int)e - 25);
  return u2f(f2u(v) | s);
}

uint16_t ora_f32_to_bf16(float x) {
  uint32_t u = f2u(x);
  uint16_t s = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(s | 0x7fffu);
  if (a == 0x7f800000u) return (uint16_t)(s | 0x7f80u);
  uint32_t c = rne_code(a, 7, 127, -126);
  if (c >= 0x7f80u) c = 0x7f80u;
  return (uint16_t)(s | c);
}

/* any_tensor.mojo:1322-1332: bf16 occupies the upper 16 bits of a float32 */
float ora_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint8_t ora_f32_to_e4m3(float x) {
  uint32_t u = f2u(x);
  uint8_t s = (uint8_t)((u >> 24) & 0x80u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return 0x7f;
  if (a == 0x7f800000u) return (uint8_t)(s | 0x7e);
  uint32_t c = rne_code(a, 3, 7, -6);
  if (c > 0x7eu) c = 0x7eu;
  return (uint8_t)(s | c);
}

float ora_e4m3_to_f32(uint8_t b) {
  int e = (b >> 3) & 0xf, m = b & 7;
  float v;
  if (e == 0)
    v = ldexpf((float)m, -9);
  else if (e == 15 && m == 7)
    return NAN;
  else
    v = ldexpf((float)(8 + m), e - 10);
  return (b & 0x80) ? -v : v;
}

uint8_t ora_f32_to_e5m2(float x) {
  uint32_t u = f2u(x);
  uint8_t s = (uint8_t)((u >> 24) & 0x80u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return 0x7f;
  if (a == 0x7f800000u) return (uint8_t)(s | 0x7b);
  uint32_t c = rne_code(a, 2, 15, -14);
  if (c > 0x7bu) c = 0x7bu;
  return (uint8_t)(s | c);
}

float ora_e5m2_to_f32(uint8_t b) {
  int e = (b >> 2) & 0x1f, m = b & 3;
  float v;
  if (e == 0)
    v = ldexpf((float)m, -16);
  else if (e == 31)
    return m ? NAN : ((b & 0x80) ? -INFINITY : INFINITY);
  else
    v = ldexpf((float)(4 + m), e - 17);
  return (b & 0x80) ? -v : v;
}

/* ------------------------------------------------------------------------ */
/* FP4 E2M1 and block scales                                                */
/* ------------------------------------------------------------------------ */

/* src/odyssey/core/types/mxfp4.mojo:51-84 (_e8m0_from_float32) */
uint8_t ora_e8m0_from_f32(float scale) {
  if (scale <= 0.0f || isnan(scale)) return 0;
  if (isinf(scale)) return 255;
  uint32_t bits = f2u(scale);
  uint8_t e = (uint8_t)((bits >> 23) & 0xff);
  uint32_t mant = bits & 0x7fffff;
  if (mant >= 0x400000u) {
    if (e < 255) e++;
  }
  return e;
}

/* mxfp4.mojo:87-112 (_e8m0_to_float32) */
float ora_e8m0_to_f32(uint8_t e) {
  if (e == 0) return 0.0f;
  if (e == 255) return INFINITY;
  return u2f((uint32_t)e << 23);
}

/* src/odyssey/core/types/nvfp4.mojo:57-81 (_e4m3_from_float32) */
uint8_t ora_e4m3_scale_from_f32(float scale) {
  if (scale <= 0.0f || isnan(scale)) return 0;
  if (isinf(scale) || scale >= 240.0f) return 0x7e;
  float a = scale > 0 ? scale : -scale;
  return ora_f32_to_e4m3(a);
}

/* mxfp4.mojo:144-224 and nvfp4.mojo:125-205 (_fp4_from_float32; the two
 * copies are identical).  Thresholds: <0.5 -> 0, <1.25 -> 1.0, <1.75 -> 1.5,
 * <2.5 -> 2.0, <3.5 -> 3.0, <5.0 -> 4.0, else 6.0 (ties round up). */
uint8_t ora_fp4_from_f32(float x, float scale) {
  if (isnan(x)) return 0x7;
  if (isinf(x)) return x > 0 ? 0x7 : 0xf;
  float scaled = x / scale;
  if (scaled == 0.0f) return 0;
  uint8_t sign = 0;
  float a = scaled;
  if (scaled < 0) {
    sign = 1;
    a = -scaled;
  }
  if (a >= 6.0f) return (uint8_t)((sign << 3) | 0x7);
  if (a < 0.5f) return (uint8_t)(sign << 3);
  uint8_t e, m;
  if (a < 1.25f) {
    e = 1; m = 0;
  } else if (a < 1.75f) {
    e = 1; m = 1;
  } else if (a < 2.5f) {
    e = 2; m = 0;
  } else if (a < 3.5f) {
    e = 2; m = 1;
  } else if (a < 5.0f) {
    e = 3; m = 0;
  } else {
    e = 3; m = 1;
  }
  return (uint8_t)((sign << 3) | (e << 1) | m);
}

/* MXFP4._fp4_stochastic_round (mxfp4.mojo:398-483; the NVFP4 copy,
 * nvfp4.mojo:386-471, is identical): bucket of |x/scale| between two E2M1
 * values (0 and 1.0 adjacent: 0.5 is never produced), probability of the
 * upper one (|x/scale| - lower) / (upper - lower), one LCG step on the low
 * 32 bits of the seed, its top 24 bits / 2^24 compared with it. */
static uint8_t fp4_stochastic_round(float x, float scale, uint64_t seed) {
  float scaled = x / scale;
  uint8_t sign = 0;
  float a = scaled;
  if (scaled < 0) {
    sign = 1;
    a = -scaled;
  }
  float lower, upper;
  uint8_t lb, ub;
  if (a < 0.5f) return (uint8_t)(sign << 3);
  else if (a < 1.0f) { lower = 0.0f; upper = 1.0f; lb = 0x0; ub = 0x2; }
  else if (a < 1.5f) { lower = 1.0f; upper = 1.5f; lb = 0x2; ub = 0x3; }
  else if (a < 2.0f) { lower = 1.5f; upper = 2.0f; lb = 0x3; ub = 0x4; }
  else if (a < 3.0f) { lower = 2.0f; upper = 3.0f; lb = 0x4; ub = 0x5; }
  else if (a < 4.0f) { lower = 3.0f; upper = 4.0f; lb = 0x5; ub = 0x6; }
  else if (a < 6.0f) { lower = 4.0f; upper = 6.0f; lb = 0x6; ub = 0x7; }
  else return (uint8_t)((sign << 3) | 0x7);
  float dist = a - lower;
  float range = upper - lower;
  float prob_up = dist / range;
  uint32_t st = (uint32_t)seed;
  st = 1103515245u * st + 12345u;
  float rv = (float)(st >> 8) / 16777216.0f;
  return (uint8_t)((sign << 3) | (rv < prob_up ? ub : lb));
}

/* MXFP4/NVFP4.from_float32 and from_float32_stochastic (mxfp4.mojo:303-396,
 * nvfp4.mojo:290-384): NaN/Inf encode against scale 1 with the unit scale
 * byte (E8M0 127 / E4M3 0x3C), zero is code 0 with the unit scale; else the
 * power-of-two scale found by doubling while |x|/scale > 6 and halving
 * while |x|/scale < 0.5 (down to 2^-127 / 2^-7), stored as E8M0 / E4M3. */
void ora_fp4_single_encode(int kind, float x, int stochastic, uint64_t seed, uint8_t* value, uint8_t* scale) {
  const int mx = kind == ORA_Q_MXFP4;
  const uint8_t unit = mx ? 127 : 0x3C;
  if (isnan(x) || isinf(x)) {
    *value = (uint8_t)(ora_fp4_from_f32(x, 1.0f) & 0xf);
    *scale = unit;
    return;
  }
  if (x == 0.0f) {
    *value = 0;
    *scale = unit;
    return;
  }
  float ax = x > 0 ? x : -x;
  float sv = 1.0f;
  int ev = 0;
  while (ax / sv > 6.0f) {
    sv *= 2.0f;
    ev++;
  }
  while (ax / sv < 0.5f && ev > (mx ? -127 : -7)) {
    sv /= 2.0f;
    ev--;
  }
  const uint8_t e = mx ? ora_e8m0_from_f32(sv) : ora_e4m3_scale_from_f32(sv);
  const float sf = mx ? ora_e8m0_to_f32(e) : ora_e4m3_to_f32(e);
  *scale = e;
  *value = stochastic ? fp4_stochastic_round(x, sf, seed) : (uint8_t)(ora_fp4_from_f32(x, sf) & 0xf);
}

float ora_fp4_single_decode(int kind, uint8_t value, uint8_t scale) {
  const float sf = kind == ORA_Q_MXFP4 ? ora_e8m0_to_f32(scale) : ora_e4m3_to_f32(scale);
  return ora_fp4_to_f32((uint8_t)(value & 0xf), sf);
}

/* mxfp4.mojo:227-268 (_fp4_to_float32) */
float ora_fp4_to_f32(uint8_t code, float scale) {
  int sign = (code >> 3) & 1, e = (code >> 1) & 3, m = code & 1;
  if (e == 0) return sign ? -0.0f : 0.0f;
  int ex = e - 1;
  float base = 1.0f + (float)m * 0.5f;
  float un = base;
  for (int i = 0; i < ex; i++) un *= 2.0f;
  float r = un * scale;
  return sign ? -r : r;
}

/* amax as in MXFP4Block/NVFP4Block.from_float32_array: `abs_val = v if
 * v >= 0 else -v; if abs_val > max_abs` (NaN never wins). */
static float block_amax(const float* v, int n) {
  float mx = 0.0f;
  for (int i = 0; i < n; i++) {
    float a = v[i] >= 0 ? v[i] : -v[i];
    if (a > mx) mx = a;
  }
  return mx;
}

/* mxfp4.mojo:709-760 (MXFP4Block.from_float32_array); nibble order:
 * element 2i -> high nibble, 2i+1 -> low nibble; 16 code bytes then the
 * E8M0 byte (tensor_dtype_conv.mojo:281-320). */
void ora_mxfp4_block_encode(const float v[32], uint8_t out[17]) {
  float amax = block_amax(v, 32);
  float sv = amax / 6.0f;
  if (sv < 1e-10f) sv = 1.0f;
  uint8_t e = ora_e8m0_from_f32(sv);
  float sf = ora_e8m0_to_f32(e);
  for (int i = 0; i < 16; i++) {
    uint8_t a = ora_fp4_from_f32(v[2 * i], sf);
    uint8_t b = ora_fp4_from_f32(v[2 * i + 1], sf);
    out[i] = (uint8_t)(((a & 0xf) << 4) | (b & 0xf));
  }
  out[16] = e;
}

void ora_mxfp4_block_decode(const uint8_t in[17], float v[32]) {
  float sf = ora_e8m0_to_f32(in[16]);
  for (int i = 0; i < 16; i++) {
    v[2 * i] = ora_fp4_to_f32((uint8_t)((in[i] >> 4) & 0xf), sf);
    v[2 * i + 1] = ora_fp4_to_f32((uint8_t)(in[i] & 0xf), sf);
  }
}

/* nvfp4.mojo:715-763 (NVFP4Block.from_float32_array); 8 code bytes then the
 * E4M3 byte (tensor_dtype_conv.mojo:321-366). */
void ora_nvfp4_block_encode(const float v[16], uint8_t out[9]) {
  float amax = block_amax(v, 16);
  float sv = amax / 6.0f;
  if (sv < 1e-10f) sv = 1.0f;
  uint8_t e = ora_e4m3_scale_from_f32(sv);
  float sf = ora_e4m3_to_f32(e);
  for (int i = 0; i < 8; i++) {
    uint8_t a = ora_fp4_from_f32(v[2 * i], sf);
    uint8_t b = ora_fp4_from_f32(v[2 * i + 1], sf);
    out[i] = (uint8_t)(((a & 0xf) << 4) | (b & 0xf));
  }
  out[8] = e;
}

void ora_nvfp4_block_decode(const uint8_t in[9], float v[16]) {
  float sf = ora_e4m3_to_f32(in[8]);
  for (int i = 0; i < 8; i++) {
    v[2 * i] = ora_fp4_to_f32((uint8_t)((in[i] >> 4) & 0xf), sf);
    v[2 * i + 1] = ora_fp4_to_f32((uint8_t)(in[i] & 0xf), sf);
  }
}

/* ------------------------------------------------------------------------ */
/* Tensor-level quantisation                                                 */
/* ------------------------------------------------------------------------ */
int64_t ora_quant_bytes(int kind, int64_t n) {
  switch (kind) {
    case ORA_Q_FP16:
    case ORA_Q_BF16:
      return 2 * n;
    case ORA_Q_FP8_E4M3:
    case ORA_Q_FP8_E5M2:
    case ORA_Q_FP8_E4M3_TENSOR:
      return n;
    case ORA_Q_MXFP4:
    case ORA_Q_MXFP4_OCP:
      return ((n + 31) / 32) * 17;
    case ORA_Q_NVFP4:
    case ORA_Q_NVFP4_TENSOR:
      return ((n + 15) / 16) * 9;
    default:
      return 0;
  }
}

/* max |x| over a tensor, NaN ignored (same compare as block_amax) */
static float tensor_amax(const float* x, int64_t n) {
  float mx = 0.0f;
#pragma omp parallel for reduction(max : mx) num_threads(ORA_NT) schedule(static)
  for (int64_t i = 0; i < n; i++) {
    float a = x[i] >= 0 ? x[i] : -x[i];
    if (a > mx) mx = a;
  }
  return mx;
}

/* Per-tensor scales (a build-side extension; the reference has none):
 * FP8 E4M3: s = amax / 448; NVFP4: s_t = amax / (448 * 6).  A scale that is
 * not a positive finite float becomes 1.0. */
static float tensor_scale(float amax, float denom) {
  float s = amax / denom;
  if (!(s > 0.0f) || isinf(s)) s = 1.0f;
  return s;
}

/* ------------------------------------------------------------------------ */
/* MXFP4 by the OCP Microscaling Formats (MX) v1.0 rule (not the reference's */
/* mxfp4.mojo rule; BASELINE configs[1] names it).  Per 32-element block:    */
/* shared exponent X = floor(log2(max|x|)) - 2 (2 = the largest E2M1         */
/* exponent), clamped to [-127, 127], stored as the E8M0 byte X + 127; each  */
/* element is x / 2^X rounded to nearest-even on the E2M1 grid {0, 0.5, 1,   */
/* 1.5, 2, 3, 4, 6} and saturated at 6, keeping the sign of x (so -0 codes  */
/* 0x8).  A block with a NaN or Inf element gets the NaN scale byte 0xFF and */
/* zero codes (this build's choice; the spec leaves it open).  All-zero      */
/* blocks take X = 0.                                                        */
/* ------------------------------------------------------------------------ */
static uint8_t e2m1_rne(float q) {
  float a = q < 0 || (q == 0 && signbit(q)) ? -q : q;
  uint8_t c;
  if (a <= 0.25f) c = 0;
  else if (a < 0.75f) c = 1;
  else if (a <= 1.25f) c = 2;
  else if (a < 1.75f) c = 3;
  else if (a <= 2.5f) c = 4;
  else if (a < 3.5f) c = 5;
  else if (a <= 5.0f) c = 6;
  else c = 7;
  return (uint8_t)((signbit(q) ? 8 : 0) | c);
}

static void mxfp4_ocp_block_encode(const float v[32], uint8_t* blk) {
  float am = 0.0f;
  int bad = 0;
  for (int i = 0; i < 32; i++) {
    if (isnan(v[i]) || isinf(v[i])) bad = 1;
    float a = fabsf(v[i]);
    if (a > am) am = a;
  }
  if (bad) {
    memset(blk, 0, 16);
    blk[16] = 0xFF;
    return;
  }
  int X = 0;
  if (am > 0.0f) {
    int e;
    frexpf(am, &e); /* am = f * 2^e, f in [0.5, 1): floor(log2 am) = e - 1 */
    X = (e - 1) - 2;
    if (X < -127) X = -127;
    if (X > 127) X = 127;
  }
  const float r = ldexpf(1.0f, -X);
  for (int i = 0; i < 16; i++) {
    uint8_t hi = e2m1_rne(v[2 * i] * r), lo = e2m1_rne(v[2 * i + 1] * r);
    blk[i] = (uint8_t)((hi << 4) | lo);
  }
  blk[16] = (uint8_t)(X + 127);
}

static void mxfp4_ocp_block_decode(const uint8_t* blk, float v[32]) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  if (blk[16] == 0xFF) {
    for (int i = 0; i < 32; i++) v[i] = NAN;
    return;
  }
  const float s = ldexpf(1.0f, (int)blk[16] - 127);
  for (int i = 0; i < 32; i++) {
    uint8_t c = (i & 1) ? (blk[i / 2] & 15) : (blk[i / 2] >> 4);
    float m = mag[c & 7] * s;
    v[i] = (c & 8) ? -m : m;
  }
}

float ora_quantize(int kind, const float* x, int64_t n, uint8_t* out) {
  float ts = 1.0f;
  switch (kind) {
    case ORA_Q_FP16: {
      uint16_t* o = (uint16_t*)out;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) o[i] = ora_f32_to_f16(x[i]);
      break;
    }
    case ORA_Q_BF16: {
      uint16_t* o = (uint16_t*)out;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) o[i] = ora_f32_to_bf16(x[i]);
      break;
    }
    case ORA_Q_FP8_E4M3:
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_f32_to_e4m3(x[i]);
      break;
    case ORA_Q_FP8_E5M2:
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_f32_to_e5m2(x[i]);
      break;
    case ORA_Q_FP8_E4M3_TENSOR: {
      ts = tensor_scale(tensor_amax(x, n), 448.0f);
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_f32_to_e4m3(x[i] / ts);
      break;
    }
    case ORA_Q_MXFP4: {
      int64_t nb = (n + 31) / 32;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t b = 0; b < nb; b++) {
        float v[32];
        for (int i = 0; i < 32; i++) {
          int64_t k = b * 32 + i;
          v[i] = k < n ? x[k] : 0.0f; /* tensor_dtype_conv.mojo:306-307 */
        }
        ora_mxfp4_block_encode(v, out + b * 17);
      }
      break;
    }
    case ORA_Q_MXFP4_OCP: {
      int64_t nb = (n + 31) / 32;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t b = 0; b < nb; b++) {
        float v[32];
        for (int i = 0; i < 32; i++) {
          int64_t k = b * 32 + i;
          v[i] = k < n ? x[k] : 0.0f;
        }
        mxfp4_ocp_block_encode(v, out + b * 17);
      }
      break;
    }
    case ORA_Q_NVFP4:
    case ORA_Q_NVFP4_TENSOR: {
      if (kind == ORA_Q_NVFP4_TENSOR) ts = tensor_scale(tensor_amax(x, n), 2688.0f);
      int64_t nb = (n + 15) / 16;
      int scaled = kind == ORA_Q_NVFP4_TENSOR;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t b = 0; b < nb; b++) {
        float v[16];
        for (int i = 0; i < 16; i++) {
          int64_t k = b * 16 + i;
          v[i] = k < n ? (scaled ? x[k] / ts : x[k]) : 0.0f;
        }
        ora_nvfp4_block_encode(v, out + b * 9);
      }
      break;
    }
    default:
      break;
  }
  return ts;
}

/* from_fp8/from_bf8 (tensor_dtype_conv.mojo:69-92,211-235), from_mxfp4 /
 * from_nvfp4 (:369-494); per-tensor kinds multiply the decoded value by the
 * stored scale. */
void ora_dequantize(int kind, const uint8_t* q, int64_t n, float ts, float* out) {
  switch (kind) {
    case ORA_Q_FP16: {
      const uint16_t* h = (const uint16_t*)q;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_f16_to_f32(h[i]);
      break;
    }
    case ORA_Q_BF16: {
      const uint16_t* h = (const uint16_t*)q;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_bf16_to_f32(h[i]);
      break;
    }
    case ORA_Q_FP8_E4M3:
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_e4m3_to_f32(q[i]);
      break;
    case ORA_Q_FP8_E5M2:
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_e5m2_to_f32(q[i]);
      break;
    case ORA_Q_FP8_E4M3_TENSOR:
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t i = 0; i < n; i++) out[i] = ora_e4m3_to_f32(q[i]) * ts;
      break;
    case ORA_Q_MXFP4: {
      int64_t nb = (n + 31) / 32;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t b = 0; b < nb; b++) {
        float v[32];
        ora_mxfp4_block_decode(q + b * 17, v);
        for (int i = 0; i < 32 && b * 32 + i < n; i++) out[b * 32 + i] = v[i];
      }
      break;
    }
    case ORA_Q_MXFP4_OCP: {
      int64_t nb = (n + 31) / 32;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t b = 0; b < nb; b++) {
        float v[32];
        mxfp4_ocp_block_decode(q + b * 17, v);
        for (int i = 0; i < 32 && b * 32 + i < n; i++) out[b * 32 + i] = v[i];
      }
      break;
    }
    case ORA_Q_NVFP4:
    case ORA_Q_NVFP4_TENSOR: {
      int64_t nb = (n + 15) / 16;
      int scaled = kind == ORA_Q_NVFP4_TENSOR;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t b = 0; b < nb; b++) {
        float v[16];
        ora_nvfp4_block_decode(q + b * 9, v);
        for (int i = 0; i < 16 && b * 16 + i < n; i++)
          out[b * 16 + i] = scaled ? v[i] * ts : v[i];
      }
      break;
    }
    default:
      break;
  }
}

/* ------------------------------------------------------------------------ */
/* GradientScaler (src/odyssey/training/mixed_precision.mojo:45-237)         */
/* ------------------------------------------------------------------------ */
void ora_scaler_init(ora_scaler* s, float initial_scale, float growth_factor,
                     float backoff_factor, int64_t growth_interval,
                     float min_scale, float max_scale) {
  s->scale = initial_scale;
  s->growth_factor = growth_factor;
  s->backoff_factor = backoff_factor;
  s->growth_interval = growth_interval;
  s->min_scale = min_scale;
  s->max_scale = max_scale;
  s->steps_since_growth = 0;
  s->num_steps = 0;
}

/* mixed_precision.mojo:184-205 */
void ora_scaler_step(ora_scaler* s) {
  s->num_steps += 1;
  s->steps_since_growth += 1;
  if (s->steps_since_growth >= s->growth_interval) {
    float ns = s->scale * s->growth_factor;
    s->scale = ns > s->max_scale ? s->max_scale : ns;
    s->steps_since_growth = 0;
  }
}

/* mixed_precision.mojo:207-221 */
void ora_scaler_backoff(ora_scaler* s) {
  float ns = s->scale * s->backoff_factor;
  if (ns >= s->min_scale) s->scale = ns;
  s->steps_since_growth = 0;
}

/* ------------------------------------------------------------------------ */
/* unscale / finite check / norm / clip                                      */
/* ------------------------------------------------------------------------ */

/* GradientScaler.unscale_gradients (mixed_precision.mojo:154-182):
 * g / full(shape, Float64(scale), g.dtype): the divisor is the scale rounded
 * to the gradient dtype; the quotient is one IEEE division rounded to the
 * gradient dtype (for FP16 a float32 division then RNE to FP16 is the
 * correctly rounded FP16 quotient).  BF16 follows the same rule (the
 * reference's BF16 division path is unimplemented). */
void ora_unscale(int dtype, const void* g, int64_t n, float scale, void* out) {
  if (dtype == ORA_F32) {
    const float* x = (const float*)g;
    float* o = (float*)out;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
    for (int64_t i = 0; i < n; i++) o[i] = x[i] / scale;
  } else if (dtype == ORA_F16) {
    const uint16_t* x = (const uint16_t*)g;
    uint16_t* o = (uint16_t*)out;
    float d = ora_f16_to_f32(ora_f32_to_f16(scale));
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
    for (int64_t i = 0; i < n; i++) o[i] = ora_f32_to_f16(ora_f16_to_f32(x[i]) / d);
  } else {
    const uint16_t* x = (const uint16_t*)g;
    uint16_t* o = (uint16_t*)out;
    float d = ora_bf16_to_f32(ora_f32_to_bf16(scale));
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
    for (int64_t i = 0; i < n; i++) o[i] = ora_f32_to_bf16(ora_bf16_to_f32(x[i]) / d);
  }
}

static inline float load_as_f32(int dtype, const void* g, int64_t i) {
  if (dtype == ORA_F32) return ((const float*)g)[i];
  if (dtype == ORA_F16) return ora_f16_to_f32(((const uint16_t*)g)[i]);
  return ora_bf16_to_f32(((const uint16_t*)g)[i]);
}

/* check_gradients_finite (mixed_precision.mojo:357-381) -> has_nan/has_inf
 * (numerical_safety.mojo:62-152); for BF16 a real isfinite test. */
int64_t ora_count_nonfinite(int dtype, const void* g, int64_t n) {
  int64_t c = 0;
#pragma omp parallel for reduction(+ : c) num_threads(ORA_NT) schedule(static)
  for (int64_t i = 0; i < n; i++) c += !isfinite(load_as_f32(dtype, g, i));
  return c;
}

/* convert_to_fp32_master (mixed_precision.mojo:240-296): exact upcast */
void ora_upcast(int dtype, const void* g, int64_t n, float* out) {
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = load_as_f32(dtype, g, i);
}

/* _norm_sq_simd_f32 (gradient_clipping.mojo:52-67): `vec * vec` in float32,
 * `reduce_add()` of each SIMD vector in float32, accumulated in float64.
 * The reference's vector width is the host's (8 lanes on AVX2, 16 on
 * AVX-512); this restatement fixes it at 8 consecutive elements (tail
 * zero-padded) with the halves-pairwise reduce_add order
 * ((q0+q4)+(q2+q6)) + ((q1+q5)+(q3+q7)).  The float64 accumulation is
 * sequential inside fixed 65536-element blocks whose sums are then added in
 * order, which is deterministic for any thread count. */
static inline float sq8(const float* g, int64_t i, int64_t n) {
  float q[8];
  for (int k = 0; k < 8; k++) {
    float x = (i + k < n) ? g[i + k] : 0.0f;
    q[k] = x * x;
  }
  float a0 = q[0] + q[4], a1 = q[1] + q[5], a2 = q[2] + q[6], a3 = q[3] + q[7];
  return (a0 + a2) + (a1 + a3);
}

double ora_sumsq_f32(const float* g, int64_t n) {
  const int64_t B = 65536;
  int64_t nb = (n + B - 1) / B;
  double* part = (double*)malloc(sizeof(double) * (size_t)(nb > 0 ? nb : 1));
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    double acc = 0.0;
    int64_t e = (b + 1) * B < n ? (b + 1) * B : n;
    for (int64_t i = b * B; i < e; i += 8) acc += (double)sq8(g, i, n);
    part[b] = acc;
  }
  double t = 0.0;
  for (int64_t b = 0; b < nb; b++) t += part[b];
  free(part);
  return t;
}

/* clip_gradients_by_global_norm (gradient_clipping.mojo:352):
 * coef = Float64(max_norm) / (Float64(total_norm) + 1e-6), applied as
 * Float32(coef).  Returns 1.0 when total_norm <= max_norm (no clipping). */
float ora_clip_coef(float norm, float max_norm) {
  if (norm > max_norm) return (float)((double)max_norm / ((double)norm + 1e-6));
  return 1.0f;
}

/* compute_gradient_norm_list + clip_gradients_by_global_norm
 * (gradient_clipping.mojo:273-368), float32 gradients, in place. */
float ora_global_norm_clip(float** grads, const int64_t* numels, int nt, float max_norm) {
  double tot = 0.0;
  for (int i = 0; i < nt; i++) tot += ora_sumsq_f32(grads[i], numels[i]);
  float norm = (float)sqrt(tot);
  if (norm > max_norm) {
    float c = (float)((double)max_norm / ((double)norm + 1e-6));
    for (int i = 0; i < nt; i++) {
      float* g = grads[i];
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
      for (int64_t k = 0; k < numels[i]; k++) g[k] = g[k] * c;
    }
  }
  return norm;
}

/* ------------------------------------------------------------------------ */
/* Optimizers.  Each line is one whole-tensor op of the reference, rounded  */
/* to the tensor dtype; hyper-parameters are Float64 rounded once to the    */
/* tensor dtype by full_like (tensor_creation.mojo:355-376).                */
/* ------------------------------------------------------------------------ */
#define DEFINE_SGD(SUF, T)                                                      \
  void ora_sgd_step_##SUF(const T* p, const T* g, const T* vel, int64_t n,      \
                          double lr, double momentum, double wd, T* out_p,      \
                          T* out_vel) {                                         \
    const T lr_t = (T)lr, mu_t = (T)momentum, wd_t = (T)wd;                     \
    const int use_wd = wd > 0.0, use_mu = momentum > 0.0;                      \
    _Pragma("omp parallel for num_threads(ORA_NT) schedule(static)")            \
    for (int64_t i = 0; i < n; i++) {                                           \
      T e = g[i];                                                               \
      if (use_wd) { /* sgd.mojo:90-95 */                                        \
        T d = wd_t * p[i];                                                      \
        e = g[i] + d;                                                           \
      }                                                                         \
      T nv = vel ? vel[i] : (T)0;                                               \
      if (use_mu) { /* sgd.mojo:99-113 */                                       \
        T s = mu_t * vel[i];                                                    \
        nv = s + e;                                                             \
        e = nv;                                                                 \
      }                                                                         \
      T u = lr_t * e; /* sgd.mojo:115-118 */                                    \
      out_p[i] = p[i] - u;                                                      \
      if (out_vel) out_vel[i] = nv;                                             \
    }                                                                           \
  }
DEFINE_SGD(f32, float)
DEFINE_SGD(f64, double)

#define DEFINE_ADAM(NAME, T, SQRT, DECOUPLED)                                   \
  void NAME(const T* p, const T* g, const T* m, const T* v, int64_t n,          \
            int64_t t, double lr, double b1, double b2, double eps, double wd,  \
            T* out_p, T* out_m, T* out_v) {                                     \
    const T b1_t = (T)b1, omb1 = (T)(1.0 - b1), b2_t = (T)b2,                   \
            omb2 = (T)(1.0 - b2);                                               \
    const T bc1 = (T)(1.0 - pow(b1, (double)t));                                \
    const T bc2 = (T)(1.0 - pow(b2, (double)t));                                \
    const T eps_t = (T)eps, lr_t = (T)lr, wd_t = (T)wd;                         \
    const int use_wd = wd > 0.0;                                                \
    _Pragma("omp parallel for num_threads(ORA_NT) schedule(static)")            \
    for (int64_t i = 0; i < n; i++) {                                           \
      T e = g[i];                                                               \
      if (!(DECOUPLED) && use_wd) { /* adam.mojo:116-121 */                     \
        T d = wd_t * p[i];                                                      \
        e = g[i] + d;                                                           \
      }                                                                         \
      T md = b1_t * m[i]; /* m = b1*m + (1-b1)*e */                             \
      T gt = omb1 * e;                                                          \
      T nm = md + gt;                                                           \
      T vd = b2_t * v[i]; /* v = b2*v + (1-b2)*(e*e) */                         \
      T g2 = e * e;                                                             \
      T g2t = omb2 * g2;                                                        \
      T nv = vd + g2t;                                                          \
      T mh = nm / bc1;                                                          \
      T vh = nv / bc2;                                                          \
      T sq = SQRT(vh);                                                          \
      T den = sq + eps_t;                                                       \
      T dir = mh / den;                                                         \
      T upd = lr_t * dir;                                                       \
      T np = p[i] - upd;                                                        \
      if ((DECOUPLED) && use_wd) { /* adamw.mojo:165-172 */                     \
        T dec = wd_t * np;                                                      \
        np = np - dec;                                                          \
      }                                                                         \
      out_p[i] = np;                                                            \
      out_m[i] = nm;                                                            \
      out_v[i] = nv;                                                            \
    }                                                                           \
  }
/* adam.mojo:42-166 */
DEFINE_ADAM(ora_adam_step_f32, float, sqrtf, 0)
DEFINE_ADAM(ora_adam_step_f64, double, sqrt, 0)
/* adamw.mojo:44-175 */
DEFINE_ADAM(ora_adamw_step_f32, float, sqrtf, 1)
DEFINE_ADAM(ora_adamw_step_f64, double, sqrt, 1)

/* lion.mojo:76-104: the momentum EMA uses beta2; the sign of the beta1
 * interpolation of the OLD momentum is the step; decoupled weight decay
 * lr*wd (one Float64 product rounded once) times the OLD params, applied
 * when wd != 0.  sign(x) is 1 for x > 0, -1 for x < 0, else 0
 * (elementwise.mojo:148-155, so NaN gives 0). */
#define DEFINE_LION(SUF, T)                                                     \
  void ora_lion_step_##SUF(const T* p, const T* g, const T* m, int64_t n,       \
                           double lr, double b1, double b2, double wd,          \
                           T* out_p, T* out_m) {                                \
    const T b2_t = (T)b2, omb2 = (T)(1.0 - b2), b1_t = (T)b1,                   \
            omb1 = (T)(1.0 - b1), lr_t = (T)lr, wdlr = (T)(wd * lr);            \
    const int use_wd = wd != 0.0;                                              \
    _Pragma("omp parallel for num_threads(ORA_NT) schedule(static)")            \
    for (int64_t i = 0; i < n; i++) {                                           \
      T a = b2_t * m[i];                                                        \
      T c = omb2 * g[i];                                                        \
      T nm = a + c;                                                             \
      T x1 = b1_t * m[i];                                                       \
      T x2 = omb1 * g[i];                                                       \
      T x = x1 + x2;                                                            \
      T u = x > (T)0 ? (T)1 : (x < (T)0 ? (T)-1 : (T)0);                        \
      T lu = lr_t * u;                                                          \
      T np = p[i] - lu;                                                         \
      if (use_wd) {                                                             \
        T d = wdlr * p[i];                                                      \
        np = np - d;                                                            \
      }                                                                         \
      out_p[i] = np;                                                            \
      out_m[i] = nm;                                                            \
    }                                                                           \
  }
DEFINE_LION(f32, float)
DEFINE_LION(f64, double)

/* rmsprop.mojo:128-175: coupled weight decay (wd > 0) into the gradient,
 * square_avg EMA, eps outside the sqrt, optional momentum buffer (a zero
 * buffer when none is given), p - lr*update. */
#define DEFINE_RMSPROP(SUF, T, SQRT)                                            \
  void ora_rmsprop_step_##SUF(const T* p, const T* g, const T* sq,              \
                              const T* buf, int64_t n, double lr, double alpha, \
                              double eps, double wd, double momentum, T* out_p, \
                              T* out_sq, T* out_buf) {                          \
    const T al = (T)alpha, oma = (T)(1.0 - alpha), eps_t = (T)eps,              \
            lr_t = (T)lr, wd_t = (T)wd, mu_t = (T)momentum;                     \
    const int use_wd = wd > 0.0, use_mu = momentum > 0.0;                      \
    _Pragma("omp parallel for num_threads(ORA_NT) schedule(static)")            \
    for (int64_t i = 0; i < n; i++) {                                           \
      T e = g[i];                                                               \
      if (use_wd) {                                                             \
        T d = wd_t * p[i];                                                      \
        e = g[i] + d;                                                           \
      }                                                                         \
      T g2 = e * e;                                                             \
      T a1 = al * sq[i];                                                        \
      T a2 = oma * g2;                                                          \
      T nsq = a1 + a2;                                                          \
      T den = SQRT(nsq) + eps_t;                                                \
      T ng = e / den;                                                           \
      T upd = ng;                                                               \
      if (use_mu) {                                                             \
        T b = buf ? buf[i] : (T)0;                                              \
        T bt = mu_t * b;                                                        \
        upd = bt + ng;                                                          \
        if (out_buf) out_buf[i] = upd;                                          \
      }                                                                         \
      T pu = lr_t * upd;                                                        \
      out_p[i] = p[i] - pu;                                                     \
      out_sq[i] = nsq;                                                          \
    }                                                                           \
  }
DEFINE_RMSPROP(f32, float, sqrtf)
DEFINE_RMSPROP(f64, double, sqrt)

/* adagrad.mojo:93-118: accum + g*g (no weight decay fold), eps outside the
 * sqrt, lr*g/den, plus wd*p outside the adaptive scaling when wd > 0. */
#define DEFINE_ADAGRAD(SUF, T, SQRT)                                            \
  void ora_adagrad_step_##SUF(const T* p, const T* g, const T* acc, int64_t n,  \
                              double lr, double eps, double wd, T* out_p,       \
                              T* out_acc) {                                     \
    const T eps_t = (T)eps, lr_t = (T)lr, wd_t = (T)wd;                         \
    const int use_wd = wd > 0.0;                                               \
    _Pragma("omp parallel for num_threads(ORA_NT) schedule(static)")            \
    for (int64_t i = 0; i < n; i++) {                                           \
      T g2 = g[i] * g[i];                                                       \
      T na = acc[i] + g2;                                                       \
      T den = SQRT(na) + eps_t;                                                 \
      T ag = g[i] / den;                                                        \
      T upd = lr_t * ag;                                                        \
      if (use_wd) {                                                             \
        T d = wd_t * p[i];                                                      \
        upd = upd + d;                                                          \
      }                                                                         \
      out_p[i] = p[i] - upd;                                                    \
      out_acc[i] = na;                                                          \
    }                                                                           \
  }
DEFINE_ADAGRAD(f32, float, sqrtf)
DEFINE_ADAGRAD(f64, double, sqrt)

/* ------------------------------------------------------------------------ */
/* The fused step, in the order of examples/mixed_precision_training.mojo:  */
/* 132-216 and examples/lenet_emnist/run_train.mojo:219-306:                 */
/* unscale -> finite check over all tensors -> [skip + backoff] -> upcast   */
/* -> global-norm clip -> optimizer -> requant -> scaler.step().            */
/* PrecisionConfig.step (precision_config.mojo:455-473) does the counters.  */
/* ------------------------------------------------------------------------ */
int ora_fused_step(ora_tensor* ts, int nt, const ora_cfg* cfg, ora_scaler* sc,
                   int64_t* step_count, int64_t* overflow_count, int64_t t,
                   ora_result* res) {
  memset(res, 0, sizeof(*res));
  if ((cfg->optimizer == ORA_ADAM || cfg->optimizer == ORA_ADAMW || cfg->optimizer == ORA_RMSPROP) && t <= 0)
    return -1;
  res->scale_used = sc->scale;
  int64_t total = 0;
  for (int i = 0; i < nt; i++) total += ts[i].numel;
  float* g32 = (float*)malloc(sizeof(float) * (size_t)(total > 0 ? total : 1));
  int64_t off = 0, nonfinite = 0;
  double sumsq = 0.0;
  for (int i = 0; i < nt; i++) {
    int64_t n = ts[i].numel;
    int dt = ts[i].grad_dtype;
    size_t esz = dt == ORA_F32 ? 4 : 2;
    void* u = malloc(esz * (size_t)(n > 0 ? n : 1));
    if (cfg->use_scaler)
      ora_unscale(dt, ts[i].grad, n, sc->scale, u);
    else
      memcpy(u, ts[i].grad, esz * (size_t)n);
    nonfinite += ora_count_nonfinite(dt, u, n);
    ora_upcast(dt, u, n, g32 + off);
    free(u);
    sumsq += ora_sumsq_f32(g32 + off, n);
    off += n;
  }
  res->nonfinite = nonfinite;
  res->sumsq = sumsq;
  res->norm = (float)sqrt(sumsq);
  res->coef = 1.0f;
  *step_count += 1;
  if (nonfinite > 0) {
    res->skipped = 1;
    if (cfg->use_scaler) {
      ora_scaler_backoff(sc);
      *overflow_count += 1;
    }
  } else {
    if (cfg->clip_enabled) {
      res->coef = ora_clip_coef(res->norm, cfg->max_norm);
      res->clipped = res->norm > cfg->max_norm;
      if (res->clipped) {
        float c = res->coef;
#pragma omp parallel for num_threads(ORA_NT) schedule(static)
        for (int64_t k = 0; k < total; k++) g32[k] = g32[k] * c;
      }
    }
    off = 0;
    for (int i = 0; i < nt; i++) {
      ora_tensor* T = &ts[i];
      int64_t n = T->numel;
      const float* g = g32 + off;
      switch (cfg->optimizer) {
        case ORA_SGD:
          ora_sgd_step_f32(T->master, g, T->s1, n, cfg->lr, cfg->momentum,
                           cfg->weight_decay, T->master, T->s1);
          break;
        case ORA_LION:
          ora_lion_step_f32(T->master, g, T->s1, n, cfg->lr, cfg->beta1, cfg->beta2, cfg->weight_decay,
                            T->master, T->s1);
          break;
        case ORA_RMSPROP:
          ora_rmsprop_step_f32(T->master, g, T->s1, T->s2, n, cfg->lr, cfg->alpha, cfg->epsilon,
                               cfg->weight_decay, cfg->momentum, T->master, T->s1, T->s2);
          break;
        case ORA_ADAGRAD:
          ora_adagrad_step_f32(T->master, g, T->s1, n, cfg->lr, cfg->epsilon, cfg->weight_decay, T->master,
                               T->s1);
          break;
        case ORA_ADAM:
          ora_adam_step_f32(T->master, g, T->s1, T->s2, n, t, cfg->lr, cfg->beta1,
                            cfg->beta2, cfg->epsilon, cfg->weight_decay, T->master,
                            T->s1, T->s2);
          break;
        default:
          ora_adamw_step_f32(T->master, g, T->s1, T->s2, n, t, cfg->lr, cfg->beta1,
                             cfg->beta2, cfg->epsilon, cfg->weight_decay, T->master,
                             T->s1, T->s2);
          break;
      }
      if (T->quant != ORA_Q_NONE && T->qout) {
        float s = ora_quantize(T->quant, T->master, n, T->qout);
        if (T->qscale) *T->qscale = s;
      }
      off += n;
    }
    if (cfg->use_scaler) ora_scaler_step(sc);
  }
  free(g32);
  res->scale_next = sc->scale;
  res->step_count = *step_count;
  res->overflow_count = *overflow_count;
  return 0;
}
