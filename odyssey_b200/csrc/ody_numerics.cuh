// ody_numerics.cuh -- device-side numerics of the mixed-precision update path.
//
// Every arithmetic operation of the reference is a separate whole-tensor op
// rounded to float32 (src/odyssey/core/arithmetic_simd.mojo:39-197,
// src/odyssey/tensor/typed/arithmetic_simd.mojo:13-125), so the kernels use
// the explicitly rounded intrinsics (__fadd_rn/__fmul_rn/__fdiv_rn/
// __fsqrt_rn); they are never contracted into FMAs and never flush
// denormals, which makes the float32 results bit-identical to the reference
// order of operations.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace ody {

enum : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };
enum : int { OPT_SGD = 0, OPT_ADAM = 1, OPT_ADAMW = 2, OPT_LION = 3, OPT_RMSPROP = 4, OPT_ADAGRAD = 5 };
enum : int {
  Q_NONE = 0,
  Q_FP16 = 1,
  Q_BF16 = 2,
  Q_FP8_E4M3 = 3,
  Q_FP8_E5M2 = 4,
  Q_FP8_E4M3_TENSOR = 5,
  Q_MXFP4 = 6,
  Q_NVFP4 = 7,
  Q_NVFP4_TENSOR = 8,
  Q_MXFP4_OCP = 9
};

// Optimizer constants, each a Float64 hyper-parameter rounded once to
// float32 as full_like does (src/odyssey/tensor/tensor_creation.mojo:355-376).
struct OptConsts {
  float lr, mu, wd;          // sgd.mojo:27-121
  float b1, omb1, b2, omb2;  // adam.mojo:123-140
  float bc1, bc2, eps;       // adam.mojo:142-163
  float alpha, omalpha;      // rmsprop.mojo:144-152
  float wdlr;                // lion.mojo:100-103: Float64(wd * lr) rounded once
  int use_wd, use_mu;
  int use_wd_nz;             // lion.mojo:100: weight_decay != 0
};

// sgd.mojo:89-118: e = g + wd*p; v' = mu*v + e; p' = p - lr*v'
__device__ __forceinline__ void sgd_elem(float& p, float g, float& vel, const OptConsts& c) {
  float e = g;
  if (c.use_wd) e = __fadd_rn(g, __fmul_rn(c.wd, p));
  if (c.use_mu) {
    vel = __fadd_rn(__fmul_rn(c.mu, vel), e);
    e = vel;
  }
  p = __fsub_rn(p, __fmul_rn(c.lr, e));
}

// adam.mojo:116-163 (DECOUPLED=false) and adamw.mojo:123-172 (true)
template <bool DECOUPLED>
__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v, const OptConsts& c) {
  float e = g;
  if (!DECOUPLED && c.use_wd) e = __fadd_rn(g, __fmul_rn(c.wd, p));
  m = __fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.omb1, e));
  v = __fadd_rn(__fmul_rn(c.b2, v), __fmul_rn(c.omb2, __fmul_rn(e, e)));
  const float mh = __fdiv_rn(m, c.bc1);
  const float vh = __fdiv_rn(v, c.bc2);
  const float den = __fadd_rn(__fsqrt_rn(vh), c.eps);
  float np = __fsub_rn(p, __fmul_rn(c.lr, __fdiv_rn(mh, den)));
  if (DECOUPLED && c.use_wd) np = __fsub_rn(np, __fmul_rn(c.wd, np));
  p = np;
}

// lion.mojo:76-104: m' = b2*m + (1-b2)*g; step = sign(b1*m + (1-b1)*g) of
// the old m (sign: 1 / -1 / 0, NaN -> 0, elementwise.mojo:148-155);
// p' = p - lr*step - (wd*lr)*p with the old p
__device__ __forceinline__ void lion_elem(float& p, float g, float& m, const OptConsts& c) {
  const float nm = __fadd_rn(__fmul_rn(c.b2, m), __fmul_rn(c.omb2, g));
  const float x = __fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.omb1, g));
  const float u = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
  float np = __fsub_rn(p, __fmul_rn(c.lr, u));
  if (c.use_wd_nz) np = __fsub_rn(np, __fmul_rn(c.wdlr, p));
  p = np;
  m = nm;
}

// rmsprop.mojo:128-175: e = g + wd*p (wd > 0); sq' = alpha*sq + (1-alpha)*e^2
// (pow(e, 2.0) as the correctly rounded e*e); n = e / (sqrt(sq') + eps);
// with momentum buf' = mu*buf + n is the update; p' = p - lr*update
__device__ __forceinline__ void rmsprop_elem(float& p, float g, float& sq, float& buf, const OptConsts& c) {
  float e = g;
  if (c.use_wd) e = __fadd_rn(g, __fmul_rn(c.wd, p));
  const float nsq = __fadd_rn(__fmul_rn(c.alpha, sq), __fmul_rn(c.omalpha, __fmul_rn(e, e)));
  const float den = __fadd_rn(__fsqrt_rn(nsq), c.eps);
  float upd = __fdiv_rn(e, den);
  if (c.use_mu) {
    buf = __fadd_rn(__fmul_rn(c.mu, buf), upd);
    upd = buf;
  }
  p = __fsub_rn(p, __fmul_rn(c.lr, upd));
  sq = nsq;
}

// adagrad.mojo:93-118: acc' = acc + g*g; update = lr * g / (sqrt(acc') + eps)
// (+ wd*p outside the adaptive scaling when wd > 0); p' = p - update
__device__ __forceinline__ void adagrad_elem(float& p, float g, float& acc, const OptConsts& c) {
  const float na = __fadd_rn(acc, __fmul_rn(g, g));
  const float den = __fadd_rn(__fsqrt_rn(na), c.eps);
  float upd = __fmul_rn(c.lr, __fdiv_rn(g, den));
  if (c.use_wd) upd = __fadd_rn(upd, __fmul_rn(c.wd, p));
  p = __fsub_rn(p, upd);
  acc = na;
}

// ---- low-precision element casts (IEEE round-to-nearest-even) -------------
__device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
  return __half_as_ushort(__float2half_rn(x));
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float((uint32_t)h << 16);
}

// float32 -> FP8 with hardware cvt (rn, satfinite); NaN is normalised to
// 0x7F so the encoding of NaN is fixed.
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  if (x != x) return 0x7f;
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ uint8_t f32_to_e5m2(float x) {
  if (x != x) return 0x7f;
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E5M2);
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3)));
}
__device__ __forceinline__ float e5m2_to_f32(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E5M2)));
}

// ---- FP4 block scales ----------------------------------------------------
// src/odyssey/core/types/mxfp4.mojo:51-84: exponent field of amax/6, +1 when
// the mantissa is >= 0.5 (round to nearest power of two), capped at 255.
__device__ __forceinline__ uint8_t e8m0_from_f32(float s) {
  if (!(s > 0.0f)) return 0;  // <= 0 or NaN
  uint32_t b = __float_as_uint(s);
  if (b == 0x7f800000u) return 255;
  uint32_t e = (b >> 23) & 0xff;
  if ((b & 0x7fffff) >= 0x400000u && e < 255) e++;
  return (uint8_t)e;
}
// mxfp4.mojo:87-112
__device__ __forceinline__ float e8m0_to_f32(uint8_t e) {
  if (e == 0) return 0.0f;
  if (e == 255) return __uint_as_float(0x7f800000u);
  return __uint_as_float((uint32_t)e << 23);
}
// src/odyssey/core/types/nvfp4.mojo:57-81
__device__ __forceinline__ uint8_t e4m3_scale_from_f32(float s) {
  if (!(s > 0.0f)) return 0;
  if (s >= 240.0f) return 0x7e;  // includes +inf
  return f32_to_e4m3(s);
}

// Block scale value (amax/6 with the 1e-10 -> 1.0 fallback of
// MXFP4Block/NVFP4Block.from_float32_array: mxfp4.mojo:733-747,
// nvfp4.mojo:738-748).
__device__ __forceinline__ float block_scale_value(float amax) {
  float s = __fdiv_rn(amax, 6.0f);
  if (s < 1e-10f) s = 1.0f;
  return s;
}

// amax compare of the reference (`abs_val = v if v >= 0 else -v; if abs_val >
// max_abs`): NaN never wins.  fmaxf drops NaN operands the same way.
__device__ __forceinline__ float amax_acc(float acc, float x) { return fmaxf(acc, fabsf(x)); }

// ---- E2M1 encode via per-scale thresholds ----------------------------------
// The reference encodes q = x / scale (IEEE division) against the ladder
// <0.5 -> 0, <1.25 -> 1.0, <1.75 -> 1.5, <2.5 -> 2.0, <3.5 -> 3.0, <5.0 -> 4.0,
// else 6.0 (mxfp4.mojo:144-224, nvfp4.mojo:125-205).  Because x -> RN(x/s) is
// monotone, each compare RN(|x|/s) >= T is exactly |x| >= X_T(s), where X_T(s)
// is the least float whose IEEE quotient reaches T.  The host computes X_T(s)
// for every representable block scale by bisection with real IEEE
// divisions, so the device needs only compares: bit-exact by construction.
// thr[0] = least |x| with RN(|x|/s) > 0 (decides the sign bit of tiny
// negatives), thr[1..6] = X_T for T = 0.5, 1.25, 1.75, 2.5, 3.5, 5.0.
// A threshold of NaN means "never" (scale = +inf).
struct __align__(16) Fp4Thr {
  float t[8];
};

// one table entry into registers with two 128-bit loads (scalar loads of
// entries e*8 + k from shared memory hit only 4 bank groups across a warp)
__device__ __forceinline__ void thr_load(const Fp4Thr* p, float t[8]) {
  const float4 a = reinterpret_cast<const float4*>(p->t)[0];
  const float4 b = reinterpret_cast<const float4*>(p->t)[1];
  t[0] = a.x; t[1] = a.y; t[2] = a.z; t[3] = a.w;
  t[4] = b.x; t[5] = b.y; t[6] = b.z; t[7] = b.w;
}

__device__ __forceinline__ uint32_t fp4_encode(float x, const float* thr, bool scale_zero) {
  const float a = fabsf(x);
  uint32_t mag = 2u * (a >= thr[1]) + (a >= thr[2]) + (a >= thr[3]) + (a >= thr[4]) +
                 (a >= thr[5]) + (a >= thr[6]);
  uint32_t sign = (x < 0.0f) && (a >= thr[0]);
  uint32_t code = (sign << 3) | mag;
  if (x != x) code = 0x7;                      // isnan(x) -> 0b0111
  if (a == __uint_as_float(0x7f800000u)) code = x > 0.0f ? 0x7u : 0xfu;  // isinf(x)
  if (scale_zero && a == 0.0f) code = 0x7;     // 0/0 = NaN -> else-branch 0b0111
  return code;
}

// mxfp4.mojo:227-268 (_fp4_to_float32): exp 0 -> +-0 (no scale multiply),
// else +-(2^(e-1) * (1 + m/2)) * scale.
__device__ __forceinline__ float fp4_decode(uint32_t code, float scale) {
  const uint32_t e = (code >> 1) & 3u, m = code & 1u;
  const bool neg = (code >> 3) & 1u;
  if (e == 0) return neg ? -0.0f : 0.0f;
  float un = m ? 1.5f : 1.0f;
  un = un * (float)(1u << (e - 1));
  float r = __fmul_rn(un, scale);
  return neg ? -r : r;
}

}  // namespace ody
