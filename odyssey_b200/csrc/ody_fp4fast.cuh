// ody_fp4fast.cuh -- FP4 (E2M1) block encoding with one thread per block.
//
// The reference encodes each element as the ladder code of q = RN(x / scale)
// (IEEE division): <0.5 -> 0, <1.25 -> 1.0, <1.75 -> 1.5, <2.5 -> 2.0,
// <3.5 -> 3.0, <5.0 -> 4.0, else 6.0, with the sign of q when q != 0
// (mxfp4.mojo:144-224, nvfp4.mojo:125-205).
//
// Two facts make this cheap:
//  1. The ladder depends only on the top 11 bits of |q|.  Its break points
//     0.5, 1.25, 1.75, 2.5, 3.5, 5.0 are the bit patterns 0x3F000000,
//     0x3FA00000, 0x3FE00000, 0x40200000, 0x40600000, 0x40A00000, all
//     multiples of 2^21, so the code is a function of bits(|q|) >> 21, which
//     clamped to [0x1F7, 0x205] takes 15 values: a shift, two integer
//     clamps and a 16-entry table lookup per element (checked over every
//     bucket against the ladder).
//  2. q itself is exact with one multiply (and two FMAs for a scale that is
//     not a power of two): MXFP4 scales are powers of two, so x * 2^-k is
//     RN(x / 2^k); for an E4M3 (or per-tensor) scale s with r = RN(1/s),
//     q0 = x*r, q = q0 + (x - q0*s)*r (the remainder exact by FMA) is the
//     correctly rounded quotient while nothing under- or overflows
//     (Markstein).  Blocks where that can fail (a non-finite element, a
//     quotient amax past 2^120, a zero scale) take the reference's
//     element-by-element division instead, and elements too small for the
//     range condition have |q| far below 0.5, where any nearby value codes
//     the same.
// The sign of a nonzero q is decided exactly with the per-scale threshold
// t0 = least |x| with RN(|x| / scale) > 0 (x <= -t0), as in the threshold
// tables.
#pragma once
#include <stdint.h>

#include "ody_numerics.cuh"

namespace ody {

// Exact division x / s with s's reciprocal r = RN(1/s) precomputed: the
// product estimate is corrected once with the exactly computed remainder
// (Markstein's correction: q0 = x*r is within one ulp, x - q0*s is exact by
// FMA, and q0 + rem*r rounded once is the correctly rounded quotient when r
// is the correctly rounded reciprocal, provided nothing under- or overflows:
// the remainder is a multiple of about ulp(x) * 2^-24, exact only while |x|
// stays above 2^-100).  Zero, non-finite and extreme magnitudes take the
// IEEE division.
__device__ __forceinline__ float div_by(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float q = __fmaf_rn(__fmaf_rn(-q0, s, x), r, q0);
  const float aq = fabsf(q0), ax = fabsf(x);
  return (aq >= 0x1p-125f && aq <= 0x1p+125f && ax >= 0x1p-100f && ax <= 0x1p+125f) ? q : __fdiv_rn(x, s);
}

// Block scale value amax / 6 (block_scale_value) through the exact
// reciprocal division.
__device__ __forceinline__ float block_scale_value_fast(float amax) {
  float v = div_by(amax, 6.0f, __frcp_rn(6.0f));
  if (v < 1e-10f) v = 1.0f;
  return v;
}


__device__ __forceinline__ uint32_t u16x2_max(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t u16x2_min(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// prmt in its default mode: a selector nibble with bit 3 set replicates the
// sign bit of the selected byte
__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(a), "r"(sel));
  return d;
}
// all ones when a <= b (false for NaN)
__device__ __forceinline__ uint32_t set_le(float a, float b) {
  uint32_t d;
  asm("set.le.u32.f32 %0, %1, %2;" : "=r"(d) : "f"(a), "f"(b));
  return d;
}
// three-input max that propagates NaN (a NaN element marks the block special)
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// q = RN(x / s) from r = RN(1/s) (valid range: see the header comment)
__device__ __forceinline__ float div_mk(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  return __fmaf_rn(__fmaf_rn(-q0, s, x), r, q0);
}

// Two quotients at once on the paired FP32 pipe (sm_100 FFMA2 / FMUL2,
// round to nearest, no flush to zero): the same operations as div_mk
// element by element, with -q0 * s written q0 * (-s), which rounds the same.
__device__ __forceinline__ float2 div_mk2(float2 x, float2 ns, float2 r) {
  const float2 q0 = __fmul2_rn(x, r);
  return __ffma2_rn(__ffma2_rn(q0, ns, x), r, q0);
}

// q[k] = div_mk(div_mk(x[k], st, rst), bs, rbs) for N (even) elements,
// |x[k]| when ABS
template <int N, bool TWO, bool ABS>
__device__ __forceinline__ void div_mk_n(const float* x, float st, float rst, float bs, float rbs, float* q) {
  const float2 nst = make_float2(-st, -st), rst2 = make_float2(rst, rst);
  const float2 nbs = make_float2(-bs, -bs), rbs2 = make_float2(rbs, rbs);
#pragma unroll
  for (int k = 0; k < N; k += 2) {
    float2 v = ABS ? make_float2(fabsf(x[k]), fabsf(x[k + 1])) : make_float2(x[k], x[k + 1]);
    if (TWO) v = div_mk2(v, nst, rst2);
    v = div_mk2(v, nbs, rbs2);
    q[k] = v.x;
    q[k + 1] = v.y;
  }
}

// Ladder index of a quotient q >= 0 (NaN and +Inf included): the ladder is
// constant on each bucket bits(q) >> 21 (its break points are the buckets
// 0x1F8, 0x1FD, 0x1FF, 0x201, 0x203, 0x205), so clamping the bucket to
// [0x1F7, 0x205] leaves 15 indices and kFp4Ladder maps them to codes.
__device__ __forceinline__ uint32_t ladder_idx(float q) {
  const int b = (int)(__float_as_uint(q) >> 21);
  return (uint32_t)(min(max(b, 0x1F7), 0x205) - 0x1F7);
}
// magnitude code per ladder index (code 1 = 0.5 is never produced)
__device__ __constant__ const uint8_t kFp4Ladder[16] = {0, 2, 2, 2, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6, 7, 7};

// 8 codes (4 bytes, element 2i in the high nibble of byte i) of quotients
// q = RN(|x| / scale) >= 0 and values x; neg_t0 = -t0 of the block's scale
// decides the sign bit; lut = the signed table of load_ladder_signed (its
// entries 0x1F7.. are the ladder codes of the clamped buckets).  The byte
// and word assembly and the sign insertion are integer multiply-adds, which
// run beside the integer pipe that the clamps use.
__device__ __forceinline__ uint32_t fp4_word(const float* q, const float* x, float neg_t0, const uint8_t* lut) {
  uint32_t w = 0;
#pragma unroll
  for (int i = 3; i >= 0; i--) {
    uint32_t b = (uint32_t)lut[0x1F7 + ladder_idx(q[2 * i])] * 16u + lut[0x1F7 + ladder_idx(q[2 * i + 1])];
    // set_le is all ones (-1) for a negative element with a nonzero quotient
    b = (uint32_t)((int)set_le(x[2 * i], neg_t0) * -128 + (int)b);
    b = (uint32_t)((int)set_le(x[2 * i + 1], neg_t0) * -8 + (int)b);
    w = w * 256u + b;
  }
  return w;
}

// Signed variant for power-of-two scales: q = RN(x / 2^k) + 0 is computed
// exactly with its sign (the "+ 0" turns -0 into +0, so a zero quotient,
// whatever the sign of x, codes 0 as in the reference's `scaled == 0.0`),
// and the bucket bits(q) >> 21 of the signed value indexes a 2048-entry
// table whose upper half holds the codes with the sign bit.
__device__ __forceinline__ void load_ladder_signed(uint8_t* lut) {
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) {
    const int b = i & 0x3FF;
    lut[i] = (uint8_t)(kFp4Ladder[min(max(b, 0x1F7), 0x205) - 0x1F7] | (i >= 0x400 ? 8 : 0));
  }
}
__device__ __forceinline__ uint32_t fp4_word_signed(const float* q, const uint8_t* lut) {
  uint32_t w = 0;
#pragma unroll
  for (int i = 3; i >= 0; i--)
    w = w * 256u + (uint32_t)lut[__float_as_uint(q[2 * i]) >> 21] * 16u + lut[__float_as_uint(q[2 * i + 1]) >> 21];
  return w;
}

// 8 codes by the reference's element-wise rule (thresholds of the block's
// scale; the special cases of NaN / Inf elements and a zero scale)
__device__ __forceinline__ uint32_t fp4_word_slow(const float* x, const float* t, bool scale_zero) {
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 4; i++)
    w |= ((fp4_encode(x[2 * i], t, scale_zero) << 4) | fp4_encode(x[2 * i + 1], t, scale_zero)) << (8 * i);
  return w;
}

// A warp's 32 blocks into its shared staging area in the output byte layout,
// with aligned 32-bit stores: each lane holds its block's NW code words and
// scale byte; four lanes fill 4 * BB bytes = BB whole words, lane r of a
// quad owning the words that start inside its bytes (its last word takes
// up to three bytes of the next lane, fetched with one shuffle).
template <int NW>
__device__ __forceinline__ void stage_blocks(uint8_t* ws, const uint32_t* cw, uint32_t sb) {
  constexpr int BB = 4 * NW + 1;
  const int lane = threadIdx.x & 31, r = lane & 3;
  const uint32_t nxt = __shfl_down_sync(0xffffffffu, cw[0], 1);
  uint32_t W[NW + 1];
#pragma unroll
  for (int k = 0; k < NW; k++) W[k] = cw[k];
  W[NW] = (sb & 0xFFu) | (nxt << 8);
  const int o0 = (4 - r) & 3;  // first owned byte offset inside the block
  uint32_t* dw = reinterpret_cast<uint32_t*>(ws) + BB * (lane >> 2) + ((BB * r + o0) >> 2);
#pragma unroll
  for (int k = 0; k < NW; k++) dw[k] = __funnelshift_r(W[k], W[k + 1], 8 * o0);
  if (r == 0) dw[NW] = W[NW];
}

// a warp's staged bytes out: 16-byte stores when the whole slice may be
// written and the destination is aligned, else bytes up to limit
__device__ __forceinline__ void flush_warp_bytes(const uint8_t* ws, uint8_t* dst, int nbytes, int64_t limit) {
  const int lane = threadIdx.x & 31;
  if (limit >= nbytes && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    for (int i = lane; i < nbytes / 16; i += 32)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(ws)[i];
  } else {
    const int m = (int)(limit < nbytes ? (limit > 0 ? limit : 0) : nbytes);
    for (int i = lane; i < m; i += 32) dst[i] = ws[i];
  }
}

// ---- asynchronous global -> shared copies (cp.async, 16 bytes per thread) --
// bytes < 16 zero-fills the rest of the 16-byte slot (bytes 0: all zeros)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
// 16-byte slot p of a staged segment, XOR-swizzled within each 128-byte row
// so that both the coalesced fill (consecutive lanes, consecutive slots) and
// the per-block read (lane l takes slots l*P .. l*P+P-1) hit distinct banks
__device__ __forceinline__ int swz16(int p) { return (p & ~7) | ((p ^ (p >> 3)) & 7); }

// Per-code constants of the NVFP4 E4M3 block scales: RN(1/scale) and t0.
struct __align__(16) NvScaleConst {
  float rcp;
  float t0;
  float scale;  // the E4M3 value itself
  float pad;
};

// ---- one NVFP4 block (16 elements) -------------------------------------
// x: the block's values (zero padded).  TS: per-tensor scale st (r_st =
// RN(1/st)) applied first, as the reference's x / s_t before the block
// encode; t0_ts[e] is then the composite t0 of E4M3 code e for this st.
// Writes the 8 code bytes (w[0], w[1]) and returns the scale byte.
// sign_fast (TS only): no nonzero element of the tensor is small enough for
// its quotient to come near zero (|x| >= 2^-124 * s_t * 2048, from the
// tensor's smallest nonzero magnitude), so every nonzero quotient is a
// normal number, exact, and carries the sign: the signed table codes it.
template <bool TS>
__device__ __forceinline__ uint32_t nv_encode_block(const float* x, float st, float rst, bool st_fast,
                                                    bool sign_fast, const float* t0_ts, const NvScaleConst* nvc,
                                                    const Fp4Thr* thr_nv, const uint8_t* lut, uint32_t* w) {
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; k += 2) am = max3_nan(am, fabsf(x[k]), fabsf(x[k + 1]));
  // am: NaN when an element is NaN, +Inf when one is infinite
  // Markstein without range guards: a tiny amax (below 2^-100) gives a
  // quotient far below the 1e-10 fallback threshold either way, and a NaN
  // or overflowing one fails the fast test below
  const float amq = TS ? div_mk(am, st, rst) : am;
  float bsv = div_mk(amq, 6.0f, 0x1.555556p-3f);  // RN(1/6)
  if (bsv < 1e-10f) bsv = 1.0f;
  const uint32_t e = e4m3_scale_from_f32(bsv);
  const bool fast = st_fast && amq <= 0x1p120f && e != 0;  // false for NaN / Inf
  if (fast) {
    const NvScaleConst c = nvc[e];
    const float bs = c.scale;
    if (TS && sign_fast) {
      float q[16];
      div_mk_n<16, true, false>(x, st, rst, bs, c.rcp, q);  // +-0 give +0
      w[0] = fp4_word_signed(q, lut);
      w[1] = fp4_word_signed(q + 8, lut);
      return e;
    }
    const float neg_t0 = -(TS ? t0_ts[e] : c.t0);
    float q[16];
    div_mk_n<16, TS, true>(x, st, rst, bs, c.rcp, q);
    w[0] = fp4_word(q, x, neg_t0, lut);
    w[1] = fp4_word(q + 8, x + 8, neg_t0, lut);
    return e;
  }
  // the reference's path: amax ignoring NaN, element-wise IEEE division
  float amr = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; k++) amr = amax_acc(amr, x[k]);
  const float amrq = TS ? div_by(amr, st, rst) : amr;
  const uint32_t er = e4m3_scale_from_f32(block_scale_value_fast(amrq));
  float t[8];
  thr_load(&thr_nv[er], t);
  float y[16];
#pragma unroll
  for (int k = 0; k < 16; k++) y[k] = TS ? __fdiv_rn(x[k], st) : x[k];
  w[0] = fp4_word_slow(y, t, er == 0);
  w[1] = fp4_word_slow(y + 8, t, er == 0);
  return er;
}

// ---- one MXFP4 block by the OCP MX v1.0 rule -----------------------------
// Shared exponent X = floor(log2(max|x|)) - 2, clamped to [-127, 127],
// stored as the E8M0 byte X + 127; elements x / 2^X (exact: a power of two)
// converted by the hardware E2M1 conversion, round to nearest even with
// saturation at +-6, sign kept.  A NaN or Inf element gives the NaN scale
// byte 0xFF and zero codes; an all-zero block X = 0.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float hi, float lo) {
  uint32_t d;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(d)
      : "f"(hi), "f"(lo));
  return d;
}
// OCP E2M1 value of a code (0, 0.5, 1, 1.5, 2, 3, 4, 6; bit 3 the sign)
// times the block scale sf (exact: a power of two, or NaN)
__device__ __forceinline__ float e2m1_ocp_decode(uint32_t code, float sf) {
  const uint32_t m = code & 7u;
  // twice the magnitude per code, as nibbles: 0, 1, 2, 3, 4, 6, 8, 12
  const float mag = (float)((0xC8643210u >> (4 * m)) & 0xFu) * 0.5f;
  const float v = __fmul_rn(mag, sf);
  return (code & 8u) ? -v : v;
}
__device__ __forceinline__ uint32_t mx_ocp_encode_block(const float* x, uint32_t* w) {
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < 32; k += 2) am = max3_nan(am, fabsf(x[k]), fabsf(x[k + 1]));
  if (!(am <= 3.4028234664e38f)) {  // NaN or Inf
#pragma unroll
    for (int i = 0; i < 4; i++) w[i] = 0;
    return 0xFF;
  }
  int X = 0;
  if (am > 0.0f) {
    const uint32_t b = __float_as_uint(am);
    const int e = (int)(b >> 23);
    // floor(log2 am): the exponent field, or for a subnormal the position of its top bit
    const int fl = e != 0 ? e - 127 : (31 - __clz(b)) - 149;
    X = min(max(fl - 2, -127), 127);
  }
  // 2^-X exactly (2^127 and the subnormal 2^-127 included)
  const float r = X <= 126 ? __uint_as_float((uint32_t)(127 - X) << 23) : __uint_as_float(0x00400000u);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint32_t wd = 0;
#pragma unroll
    for (int k = 3; k >= 0; k--)
      wd = wd * 256u + cvt_e2m1x2(__fmul_rn(x[8 * i + 2 * k], r), __fmul_rn(x[8 * i + 2 * k + 1], r));
    w[i] = wd;
  }
  return (uint32_t)(X + 127);
}

// ---- one MXFP4 block (32 elements) --------------------------------------
// Writes the 16 code bytes (w[0..3]) and returns the E8M0 scale byte.
// lut_s: the signed table of load_ladder_signed
__device__ __forceinline__ uint32_t mx_encode_block(const float* x, const Fp4Thr* thr_mx, const uint8_t* lut_s,
                                                    uint32_t* w) {
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < 32; k += 2) am = max3_nan(am, fabsf(x[k]), fabsf(x[k + 1]));
  const uint32_t e = e8m0_from_f32(block_scale_value_fast(am));
  if (am <= 0x1p127f && e >= 1 && e <= 254) {  // finite elements, a finite nonzero scale
    // 1 / 2^(e-127) exactly (2^-127 is subnormal)
    const float r = e <= 253 ? __uint_as_float((254u - e) << 23) : __uint_as_float(0x00400000u);
    float q[32];
    // the products paired; "+ 0" (-0 to +0) stays scalar, as the paired
    // add of a constant zero may be folded away
    const float2 r2 = make_float2(r, r);
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      const float2 v = __fmul2_rn(make_float2(x[k], x[k + 1]), r2);
      q[k] = __fadd_rn(v.x, 0.0f);
      q[k + 1] = __fadd_rn(v.y, 0.0f);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) w[i] = fp4_word_signed(q + 8 * i, lut_s);
    return e;
  }
  float amr = 0.0f;
#pragma unroll
  for (int k = 0; k < 32; k++) amr = amax_acc(amr, x[k]);
  const uint32_t er = e8m0_from_f32(block_scale_value_fast(amr));
  float t[8];
  thr_load(&thr_mx[er], t);
#pragma unroll
  for (int i = 0; i < 4; i++) w[i] = fp4_word_slow(x + 8 * i, t, false);
  return er;
}

}  // namespace ody
