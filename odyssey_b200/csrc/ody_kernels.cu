// ody_kernels.cu -- sm_100a kernels of the fused mixed-precision step.
//
// Pass structure of one step (all passes stream HBM; no tensor cores):
//   pass 1  stats_kernel    grads -> unscale, isfinite count, sum of float32
//                           squares in float64 (per-CTA partials, fixed-order
//                           final sum in the last CTA -> deterministic), and
//                           the GradScaler / clip decision in device memory.
//   pass 2  update_kernel   chunk-table multi-tensor apply: unscale, clip,
//                           SGD / Adam / AdamW on float32 master + states,
//                           direct requant (FP16/BF16/FP8/MXFP4/NVFP4) and the
//                           per-tensor amax of the new master for the
//                           per-tensor-scaled kinds.
//   pass 3  requant_kernel  FP8-E4M3 and NVFP4 with a per-tensor scale, which
//                           need the whole tensor's amax first.
// Standalone quantise / dequantise / single-op kernels live at the end.
#include <math.h>
#include <stdio.h>

#include <algorithm>

#include "ody_internal.h"
#include "ody_fp4fast.cuh"

namespace ody {

// ---------------------------------------------------------------------------
// FP4 threshold tables (see fp4_encode in ody_numerics.cuh).  Index: the
// E8M0 byte (MXFP4) or the E4M3 byte (NVFP4) of the block scale.
// ---------------------------------------------------------------------------
__device__ Fp4Thr g_thr_mx[256];
__device__ Fp4Thr g_thr_nv[128];
__device__ NvScaleConst g_nv_const[128];  // RN(1/scale) and t0 per E4M3 scale code

static float host_bits(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}

// least float x >= 0 with RN(x / s) >= T (IEEE float division on the host);
// NaN when no float reaches T.
static float host_threshold(float s, float T) {
  auto reaches = [&](uint32_t xb) {
    volatile float x = host_bits(xb);
    volatile float q = x / s;
    return q >= T;
  };
  uint32_t lo = 0, hi = 0x7f800000u;
  if (!reaches(hi)) return host_bits(0x7fc00000u);
  if (reaches(lo)) return 0.0f;
  while (hi - lo > 1) {
    uint32_t mid = lo + (hi - lo) / 2;
    if (reaches(mid))
      hi = mid;
    else
      lo = mid;
  }
  return host_bits(hi);
}

static void host_fill_thr(float s, Fp4Thr* t) {
  const float T[7] = {host_bits(1u), 0.5f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
  for (int k = 0; k < 7; k++) t->t[k] = host_threshold(s, T[k]);
  t->t[7] = 0.0f;
}

static float host_e8m0_to_f32(int e) {
  if (e == 0) return 0.0f;
  if (e == 255) return host_bits(0x7f800000u);
  return host_bits((uint32_t)e << 23);
}

static float host_e4m3_to_f32(int b) {
  int e = (b >> 3) & 0xf, m = b & 7;
  if (e == 0) return ldexpf((float)m, -9);
  return ldexpf((float)(8 + m), e - 10);
}

static Fp4Thr h_thr_mx[256], h_thr_nv[128];
static NvScaleConst h_nv_const[128];
static bool h_thr_ready = false;
static bool d_thr_ready[64] = {false};

void upload_fp4_tables(int device) {
  if (!h_thr_ready) {
    for (int e = 0; e < 256; e++) host_fill_thr(host_e8m0_to_f32(e), &h_thr_mx[e]);
    for (int b = 0; b < 128; b++) host_fill_thr(b == 127 ? 0.0f : host_e4m3_to_f32(b), &h_thr_nv[b]);
    for (int b = 0; b < 128; b++) {
      volatile float s = b == 127 ? 0.0f : host_e4m3_to_f32(b);
      h_nv_const[b].rcp = 1.0f / s;  // IEEE division on the host: RN(1/s)
      h_nv_const[b].t0 = h_thr_nv[b].t[0];
      h_nv_const[b].scale = s;
      h_nv_const[b].pad = 0.0f;
    }
    h_thr_ready = true;
  }
  if (device >= 0 && device < 64 && !d_thr_ready[device]) {
    cudaMemcpyToSymbol(g_thr_mx, h_thr_mx, sizeof(h_thr_mx));
    cudaMemcpyToSymbol(g_thr_nv, h_thr_nv, sizeof(h_thr_nv));
    cudaMemcpyToSymbol(g_nv_const, h_nv_const, sizeof(h_nv_const));
    d_thr_ready[device] = true;
  }
}

__device__ __forceinline__ void load_thr_smem(Fp4Thr* s_mx, Fp4Thr* s_nv) {
  float* dm = reinterpret_cast<float*>(s_mx);
  float* dn = reinterpret_cast<float*>(s_nv);
  const float* gm = reinterpret_cast<const float*>(g_thr_mx);
  const float* gn = reinterpret_cast<const float*>(g_thr_nv);
  for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) dm[i] = gm[i];
  for (int i = threadIdx.x; i < 128 * 8; i += blockDim.x) dn[i] = gn[i];
}

// ---------------------------------------------------------------------------
// Gradient loading + unscale (GradientScaler.unscale_gradients,
// src/odyssey/training/mixed_precision.mojo:154-182): g / full(F64(scale),
// g.dtype) -- divisor rounded to the gradient dtype, quotient rounded to the
// gradient dtype, then the exact upcast to float32 (convert_to_fp32_master).
// ---------------------------------------------------------------------------
template <int GDT>
__device__ __forceinline__ float unscale_divisor(float scale) {
  if (GDT == DT_F16) return f16_bits_to_f32(f32_to_f16_bits(scale));
  if (GDT == DT_BF16) return bf16_bits_to_f32(f32_to_bf16_bits(scale));
  return scale;
}

// Division by a power of two equals multiplication by its exact reciprocal
// (both are the single correct rounding of the same real number).
struct Divisor {
  float d, r;
  bool pow2;
};
__device__ __forceinline__ Divisor make_divisor(float d) {
  Divisor v;
  v.d = d;
  uint32_t b = __float_as_uint(d);
  uint32_t e = (b >> 23) & 0xff;
  v.pow2 = ((b & 0x807fffffu) == 0) && e >= 1 && e <= 254;
  v.r = v.pow2 ? __fdiv_rn(1.0f, d) : 0.0f;
  return v;
}
__device__ __forceinline__ float divide(float x, const Divisor& v) {
  return v.pow2 ? __fmul_rn(x, v.r) : __fdiv_rn(x, v.d);
}

// Fast unscale for power-of-two divisors.  A bfloat16 (or float32) value
// times an exact power of two is exact in float32 unless the product is
// float32-subnormal, so only such tiny products need the rounding back to the
// gradient dtype (float16 always rounds: its normal range is narrower).
template <int GDT>
__device__ __forceinline__ float unscale_elem(float x, const Divisor& dv) {
  if (GDT == DT_F32) return divide(x, dv);
  if (GDT == DT_BF16 && dv.pow2) {
    float q = __fmul_rn(x, dv.r);
    if (fabsf(q) < 1.17549435e-38f) q = bf16_bits_to_f32(f32_to_bf16_bits(q));
    return q;
  }
  const float q = divide(x, dv);
  return GDT == DT_F16 ? f16_bits_to_f32(f32_to_f16_bits(q)) : bf16_bits_to_f32(f32_to_bf16_bits(q));
}

// raw gradient bits of 8 consecutive elements (one or two 16-byte loads)
struct Raw8 {
  uint4 a, b;
};

template <int GDT>
__device__ __forceinline__ Raw8 ld_raw8(const void* g, int64_t e0) {
  Raw8 r;
  if (GDT == DT_F32) {
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(g) + e0);
    r.a = __ldcs(p);
    r.b = __ldcs(p + 1);
  } else {
    r.a = __ldcs(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(g) + e0));
    r.b = make_uint4(0, 0, 0, 0);
  }
  return r;
}

// exact upcast of the raw bits to float32
template <int GDT>
__device__ __forceinline__ void unpack8(const Raw8& r, float out[8]) {
  if (GDT == DT_F32) {
    out[0] = __uint_as_float(r.a.x); out[1] = __uint_as_float(r.a.y);
    out[2] = __uint_as_float(r.a.z); out[3] = __uint_as_float(r.a.w);
    out[4] = __uint_as_float(r.b.x); out[5] = __uint_as_float(r.b.y);
    out[6] = __uint_as_float(r.b.z); out[7] = __uint_as_float(r.b.w);
  } else {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      if (GDT == DT_BF16) {
        out[2 * k] = __uint_as_float(w[k] << 16);
        out[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
      } else {
        out[2 * k] = f16_bits_to_f32((uint16_t)(w[k] & 0xffffu));
        out[2 * k + 1] = f16_bits_to_f32((uint16_t)(w[k] >> 16));
      }
    }
  }
}

template <int GDT>
__device__ __forceinline__ void unscale8(float v[8], bool use_scaler, const Divisor& dv) {
  if (GDT == DT_BF16 && use_scaler && dv.pow2) {
    // exact products; only float32-subnormal ones need the bfloat16 rounding,
    // tested once for the 8 values
    float mn = 3.0e38f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      v[k] = __fmul_rn(v[k], dv.r);
      mn = fminf(mn, fabsf(v[k]));
    }
    if (mn < 1.17549435e-38f) {
#pragma unroll
      for (int k = 0; k < 8; k++)
        if (fabsf(v[k]) < 1.17549435e-38f) v[k] = bf16_bits_to_f32(f32_to_bf16_bits(v[k]));
    }
    return;
  }
  if (use_scaler) {
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = unscale_elem<GDT>(v[k], dv);
  }
}

template <int GDT>
__device__ __forceinline__ void grad8(const void* g, int64_t e0, bool use_scaler, const Divisor& dv,
                                      float out[8]) {
  unpack8<GDT>(ld_raw8<GDT>(g, e0), out);
  unscale8<GDT>(out, use_scaler, dv);
}

// Sum of the float32 squares of 8 consecutive elements, reduced in float32
// as a SIMD reduce_add of width 8 (halves added pairwise), which is how the
// reference's _norm_sq_simd_f32 (gradient_clipping.mojo:52-67) reduces each
// vector before accumulating it in float64.
__device__ __forceinline__ float sq8(const float v[8]) {
  float q[8];
#pragma unroll
  for (int k = 0; k < 8; k++) q[k] = __fmul_rn(v[k], v[k]);
  const float a0 = __fadd_rn(q[0], q[4]), a1 = __fadd_rn(q[1], q[5]);
  const float a2 = __fadd_rn(q[2], q[6]), a3 = __fadd_rn(q[3], q[7]);
  return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}

__device__ __forceinline__ bool is_finite_f(float x) { return fabsf(x) < __uint_as_float(0x7f800000u); }

// ---------------------------------------------------------------------------
// The GradientScaler / PrecisionConfig.step decision (mixed_precision.mojo:
// 184-221, precision_config.mojo:455-473) plus the global-norm clip
// coefficient (gradient_clipping.mojo:273-368).
// ---------------------------------------------------------------------------
__device__ void decide(double sumsq, int64_t nonfinite, DevScaler* sc, const DecideParams& dp,
                       Decision* out) {
  Decision r;
  memset(&r, 0, sizeof(r));
  r.sumsq = sumsq;
  r.nonfinite = nonfinite;
  r.norm = __double2float_rn(__dsqrt_rn(sumsq));
  r.scale_used = sc->scale;
  r.coef = 1.0f;
  sc->step_count += 1;
  if (nonfinite > 0) {
    r.skip = 1;
    if (dp.use_scaler) {
      float ns = __fmul_rn(sc->scale, dp.backoff_factor);
      if (ns >= dp.min_scale) sc->scale = ns;
      sc->steps_since_growth = 0;
      sc->overflow_count += 1;
    }
  } else {
    if (dp.clip_enabled && r.norm > dp.max_norm) {
      r.clipped = 1;
      r.coef = __double2float_rn(__ddiv_rn((double)dp.max_norm, __dadd_rn((double)r.norm, 1e-6)));
    }
    if (dp.use_scaler) {
      sc->num_steps += 1;
      sc->steps_since_growth += 1;
      if (sc->steps_since_growth >= dp.growth_interval) {
        float ns = __fmul_rn(sc->scale, dp.growth_factor);
        sc->scale = ns > dp.max_scale ? dp.max_scale : ns;
        sc->steps_since_growth = 0;
      }
    }
  }
  r.scale_next = sc->scale;
  r.step_count = sc->step_count;
  r.overflow_count = sc->overflow_count;
  r.scaler_num_steps = sc->num_steps;
  r.steps_since_growth = sc->steps_since_growth;
  *out = r;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum of (double, int64); result valid in thread 0.
__device__ __forceinline__ void block_sum2(double& s, long long& c) {
  __shared__ double sd[32];
  __shared__ long long sc[32];
  s = warp_sum(s);
  c = warp_sum(c);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sd[w] = s;
    sc[w] = c;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    s = l < nw ? sd[l] : 0.0;
    c = l < nw ? sc[l] : 0;
    s = warp_sum(s);
    c = warp_sum(c);
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Pass 1: gradient statistics and the step decision.
// ---------------------------------------------------------------------------
struct StatsArgs {
  const void* grad;
  int64_t n;  // multiple of 8
  int use_scaler;
  DevScaler* scaler;
  StatsPartial* partials;
  unsigned* ticket;
  int world_mode;        // 0: decide here; 1: write local_stats for the allgather
  double* local_stats;   // [2]: nonfinite (as double), sumsq
  DecideParams dp;
  Decision* dec;
  uint32_t* amax_slots;  // zeroed for pass 2
  uint32_t* sync;        // job ticket + per-tensor done counts, zeroed for pass 2
  int ntensors;
};

template <int GDT>
__device__ __forceinline__ void stats_raw8(const Raw8& r, bool use_scaler, const Divisor& dv, double& acc,
                                           long long& bad) {
  float v[8];
  unpack8<GDT>(r, v);
  if (GDT == DT_BF16 && use_scaler && dv.pow2) {
    // a bfloat16 times an exact power of two: exact unless float32-subnormal,
    // and a subnormal (or its bfloat16 rounding) squares to 0 in float32, so
    // the rounding back to bfloat16 cannot change a square or a finiteness
    // test and is skipped here (the update pass does it)
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = __fmul_rn(v[k], dv.r);
  } else {
    unscale8<GDT>(v, use_scaler, dv);
  }
  const float s = sq8(v);
  // a non-finite square sum means a NaN/Inf element or squares that overflow
  // float32; only then are the elements counted one by one
  if (!is_finite_f(s)) {
#pragma unroll
    for (int k = 0; k < 8; k++) bad += !is_finite_f(v[k]);
  }
  acc += (double)s;
}

__device__ __forceinline__ void stats_finish(const StatsArgs& a, double acc_all, long long bad);

template <int GDT>
__global__ void __launch_bounds__(kThreads, 4) stats_kernel(StatsArgs a) {
  // the apply kernel is launched as this grid's programmatic dependent: its
  // CTAs may start their prologue now and wait (griddepcontrol.wait) for
  // this grid's completion and memory flush before reading anything it writes
  asm volatile("griddepcontrol.launch_dependents;");
  const Divisor dv = make_divisor(unscale_divisor<GDT>(a.scaler->scale));
  constexpr int U = 4;
  double acc[U] = {0.0, 0.0, 0.0, 0.0};
  long long bad = 0;
  const int64_t ngroups = a.n / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (U - 1) * stride < ngroups; i += U * stride) {
    Raw8 r[U];
#pragma unroll
    for (int u = 0; u < U; u++) r[u] = ld_raw8<GDT>(a.grad, (i + u * stride) * 8);
#pragma unroll
    for (int u = 0; u < U; u++) stats_raw8<GDT>(r[u], a.use_scaler, dv, acc[u], bad);
  }
  for (; i < ngroups; i += stride) stats_raw8<GDT>(ld_raw8<GDT>(a.grad, i * 8), a.use_scaler, dv, acc[0], bad);
  stats_finish(a, (acc[0] + acc[1]) + (acc[2] + acc[3]), bad);
}

// The CTA's partial, and in the last CTA to finish the fixed-order reduction
// of all partials and the step decision (or the local pair for the
// allgather).
__device__ __forceinline__ void stats_finish(const StatsArgs& a, double acc_all, long long bad) {
  block_sum2(acc_all, bad);
  __shared__ bool last;
  if (threadIdx.x == 0) {
    a.partials[blockIdx.x].sumsq = acc_all;
    a.partials[blockIdx.x].nonfinite = bad;
    __threadfence();
    unsigned t = atomicAdd(a.ticket, 1u);
    last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // fixed-order reduction of the per-CTA partials -> deterministic sum
  double s = 0.0;
  long long c = 0;
  for (int j = threadIdx.x; j < (int)gridDim.x; j += blockDim.x) {
    s += __ldcg(&a.partials[j].sumsq);
    c += __ldcg(reinterpret_cast<const long long*>(&a.partials[j].nonfinite));
  }
  block_sum2(s, c);
  for (int j = threadIdx.x; j < a.ntensors; j += blockDim.x) a.amax_slots[j] = 0u;
  for (int j = threadIdx.x; j < a.ntensors + 1; j += blockDim.x) a.sync[j] = 0u;
  if (threadIdx.x == 0) {
    *a.ticket = 0u;
    if (a.world_mode == 0) {
      decide(s, c, a.scaler, a.dp, a.dec);
    } else {
      a.local_stats[0] = (double)c;
      a.local_stats[1] = s;
    }
  }
}

int stats_grid(int device) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms * 4;
}

cudaError_t launch_stats(int gdt, const void* grad, int64_t n, int use_scaler, DevScaler* scaler,
                         StatsPartial* partials, int grid, unsigned* ticket, int world_mode,
                         double* local_stats, const DecideParams& dp, Decision* dec,
                         uint32_t* amax_slots, uint32_t* sync, int ntensors, cudaStream_t st) {
  StatsArgs a{grad, n, use_scaler, scaler, partials, ticket, world_mode, local_stats, dp, dec,
              amax_slots, sync, ntensors};
  if (gdt == DT_F32)
    stats_kernel<DT_F32><<<grid, kThreads, 0, st>>>(a);
  else if (gdt == DT_F16)
    stats_kernel<DT_F16><<<grid, kThreads, 0, st>>>(a);
  else
    stats_kernel<DT_BF16><<<grid, kThreads, 0, st>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Data-parallel gradients: reduce-scatter fused with pass 1.  Every rank
// holds a full-model gradient buffer (its own backward's output) in the
// flat, 64-element-padded global layout; peers[q] is rank q's buffer mapped
// into this process (CUDA IPC; this rank's own at q = rank).  This rank's
// shard is the contiguous range [shard_off, shard_off + n) of that layout,
// laid out exactly like its local gradient arena.  Each group of 8
// gradients is read from every rank over NVLink (peer loads), summed in
// float32 in rank order (one rounding per add, so the result is the same on
// every run and every rank count split), rounded once to the gradient dtype
// and stored into the local arena, and its unscale / finiteness / square-sum
// statistics are taken on the stored value, as pass 1 would.  The ranks'
// readiness is ordered by an NCCL collective before this kernel, and no
// rank overwrites its buffer before the stats allgather after it, which
// needs every rank's kernel finished.
// ---------------------------------------------------------------------------
struct RsArgs {
  const void* const* peers;
  int world;
  int64_t shard_off;
  void* out;
};

template <int GDT>
__device__ __forceinline__ Raw8 pack8(const float v[8]) {
  Raw8 r;
  if (GDT == DT_F32) {
    r.a = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
    r.b = make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7]));
  } else {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t lo = GDT == DT_BF16 ? f32_to_bf16_bits(v[2 * k]) : f32_to_f16_bits(v[2 * k]);
      const uint32_t hi = GDT == DT_BF16 ? f32_to_bf16_bits(v[2 * k + 1]) : f32_to_f16_bits(v[2 * k + 1]);
      w[k] = lo | (hi << 16);
    }
    r.a = make_uint4(w[0], w[1], w[2], w[3]);
    r.b = make_uint4(0, 0, 0, 0);
  }
  return r;
}

template <int GDT>
__device__ __forceinline__ void st_raw8(void* g, int64_t e0, const Raw8& r) {
  if (GDT == DT_F32) {
    uint4* p = reinterpret_cast<uint4*>(reinterpret_cast<float*>(g) + e0);
    p[0] = r.a;
    p[1] = r.b;
  } else {
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(g) + e0) = r.a;
  }
}

// G groups of 8 gradients from each of up to R ranks (R <= 4): all G*R loads
// are issued before the first add, so that enough remote reads are in
// flight to cover the NVLink latency; the adds stay in rank order.  With 8
// ranks (G = 1) the ranks come in two batches of four.  Each reduced group
// is stored and its statistics taken at once.
template <int GDT, int R, int G>
__device__ __forceinline__ void reduce_groups(const RsArgs& rs, int64_t e0, int64_t stride_el, bool use_scaler,
                                              const Divisor& dv, double& acc_sq, long long& bad) {
  constexpr int RB = R < 4 ? R : 4;  // ranks per batch
  float acc[G][8];
#pragma unroll
  for (int q0 = 0; q0 < R; q0 += RB) {
    Raw8 raw[G][RB];
#pragma unroll
    for (int q = 0; q < RB; q++)
#pragma unroll
      for (int u = 0; u < G; u++)
        if (q0 + q < rs.world) raw[u][q] = ld_raw8<GDT>(rs.peers[q0 + q], rs.shard_off + e0 + u * stride_el);
#pragma unroll
    for (int u = 0; u < G; u++) {
#pragma unroll
      for (int q = 0; q < RB; q++) {
        if (q0 + q < rs.world) {
          float v[8];
          unpack8<GDT>(raw[u][q], v);
#pragma unroll
          for (int k = 0; k < 8; k++) acc[u][k] = (q0 + q == 0) ? v[k] : __fadd_rn(acc[u][k], v[k]);
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < G; u++) {
    const Raw8 r = pack8<GDT>(acc[u]);
    st_raw8<GDT>(rs.out, e0 + u * stride_el, r);
    stats_raw8<GDT>(r, use_scaler, dv, acc_sq, bad);
  }
}

// R: the rank count rounded up to a power of two (1, 2, 4, 8); G = 4 / R
// groups per thread per round (at least 1): four raw loads in flight
template <int GDT, int R>
__global__ void __launch_bounds__(kThreads, 4) rs_stats_kernel(StatsArgs a, RsArgs rs) {
  constexpr int G = R >= 4 ? 1 : 4 / R;
  const Divisor dv = make_divisor(unscale_divisor<GDT>(a.scaler->scale));
  double acc = 0.0;
  long long bad = 0;
  const int64_t ngroups = a.n / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (G - 1) * stride < ngroups; i += G * stride)
    reduce_groups<GDT, R, G>(rs, i * 8, stride * 8, a.use_scaler, dv, acc, bad);
  for (; i < ngroups; i += stride) reduce_groups<GDT, R, 1>(rs, i * 8, stride * 8, a.use_scaler, dv, acc, bad);
  stats_finish(a, acc, bad);
}

template <int GDT>
static void launch_rs_gdt(int world, int grid, const StatsArgs& a, const RsArgs& rs, cudaStream_t st) {
  if (world <= 1)
    rs_stats_kernel<GDT, 1><<<grid, kThreads, 0, st>>>(a, rs);
  else if (world <= 2)
    rs_stats_kernel<GDT, 2><<<grid, kThreads, 0, st>>>(a, rs);
  else if (world <= 4)
    rs_stats_kernel<GDT, 4><<<grid, kThreads, 0, st>>>(a, rs);
  else
    rs_stats_kernel<GDT, 8><<<grid, kThreads, 0, st>>>(a, rs);
}

cudaError_t launch_rs_stats(int gdt, const void* const* peers, int world, int64_t shard_off, void* grad, int64_t n,
                            int use_scaler, DevScaler* scaler, StatsPartial* partials, int grid, unsigned* ticket,
                            int world_mode, double* local_stats, const DecideParams& dp, Decision* dec,
                            uint32_t* amax_slots, uint32_t* sync, int ntensors, cudaStream_t st) {
  if (world < 1 || world > 8) return cudaErrorInvalidValue;
  StatsArgs a{grad, n, use_scaler, scaler, partials, ticket, world_mode, local_stats, dp, dec,
              amax_slots, sync, ntensors};
  RsArgs rs{peers, world, shard_off, grad};
  if (gdt == DT_F32)
    launch_rs_gdt<DT_F32>(world, grid, a, rs, st);
  else if (gdt == DT_F16)
    launch_rs_gdt<DT_F16>(world, grid, a, rs, st);
  else
    launch_rs_gdt<DT_BF16>(world, grid, a, rs, st);
  return cudaGetLastError();
}

// Multi-GPU: the per-rank {nonfinite, sumsq} pairs arrive in rank order from
// an allgather; summing them in rank order gives every rank the identical
// decision.
__global__ void finalize_kernel(const double* gathered, int world, DevScaler* sc, DecideParams dp,
                                Decision* dec, uint32_t* amax_slots, int ntensors) {
  asm volatile("griddepcontrol.launch_dependents;");
  for (int j = threadIdx.x; j < ntensors; j += blockDim.x) amax_slots[j] = 0u;
  if (threadIdx.x == 0) {
    double c = 0.0, s = 0.0;
    for (int r = 0; r < world; r++) {
      c += gathered[2 * r];
      s += gathered[2 * r + 1];
    }
    decide(s, (int64_t)c, sc, dp, dec);
  }
}

cudaError_t launch_finalize(const double* gathered, int world, DevScaler* scaler,
                            const DecideParams& dp, Decision* dec, uint32_t* amax_slots,
                            int ntensors, cudaStream_t st) {
  finalize_kernel<<<1, 256, 0, st>>>(gathered, world, scaler, dp, dec, amax_slots, ntensors);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Re-quantisation helpers shared by passes 2 and 3 and the standalone
// quantiser.  Lane l of a warp holds elements [8l, 8l+8) of the warp's 256-
// element slice of a 2048-element tile; MXFP4 blocks span 4 lanes, NVFP4
// blocks 2 lanes.  Each warp stages its slice's codes in its own piece of
// shared memory in the reference's AoS block layout
// (tensor_dtype_conv.mojo:281-366: code bytes with element 2i in the high
// nibble, then the scale byte) and writes it out with 16-byte (NVFP4, 144 B
// per warp) or 8-byte (MXFP4, 136 B per warp) stores; no CTA-wide barrier.
// ---------------------------------------------------------------------------
constexpr int kWarpStage = 288;  // bytes of shared memory per warp (32 NVFP4 blocks)
constexpr int kNvWarpBytes = 144;
constexpr int kMxWarpBytes = 136;

// 1 for a block whose codes need the reference's special cases (a NaN or
// +-Inf element, a zero NVFP4 scale, an infinite MXFP4 scale); x*0 is NaN
// exactly for non-finite x.
__device__ __forceinline__ bool any_nonfinite8(const float v[8]) {
  float z = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; k++) z = __fmaf_rn(v[k], 0.0f, z);
  return z != z;
}

// the threshold ladder without special cases (finite x, positive finite scale)
// t[1..6] are sorted (a "never" threshold is NaN and sits at the top, where
// a >= NaN is false as for +Inf), so the count of t[1..6] at or below |x| is
// found with three compares: t[3], then t[5] or t[2], then t[6], t[4] or t[1].
// The magnitude code counts t[1] twice (code 1 is never produced).
__device__ __forceinline__ uint32_t fp4_encode_plain(float x, const float* t) {
  const float a = fabsf(x);
  const bool s1 = a >= t[3];
  const bool s2 = a >= (s1 ? t[5] : t[2]);
  const uint32_t base = s1 ? (s2 ? 5u : 3u) : (s2 ? 1u : 0u);
  const uint32_t c = base + (a >= (s1 ? (s2 ? t[6] : t[4]) : t[1]));
  const uint32_t mag = c + (c != 0u);
  return ((uint32_t)((x < 0.0f) && (a >= t[0])) << 3) | mag;
}

// One lane's 8 elements of a warp's slice (lane pairs form an NVFP4 block,
// lane quads an MXFP4 block): the block scale from the shuffled amax, then
// the codes by the exact-quotient table lookup of ody_fp4fast.cuh (MXFP4:
// x * 2^-k with the sign in the table; NVFP4: the Markstein quotient and the
// t0 sign rule), or by the threshold compares where that range does not
// hold, or by the reference's special cases for non-finite elements and a
// zero scale.
template <bool MX>
__device__ __forceinline__ void stage_fp4(const float v[8], uint8_t* ws, const Fp4Thr* thr, const uint8_t* lut) {
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; k++) am = amax_acc(am, v[k]);
  am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
  if (MX) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
  const uint8_t e = MX ? e8m0_from_f32(block_scale_value_fast(am)) : e4m3_scale_from_f32(block_scale_value_fast(am));
  const bool z = !MX && e == 0;
  const bool special = z || (MX && e == 255) || any_nonfinite8(v);
  const int lane = threadIdx.x & 31;
  const int blk = MX ? (lane >> 2) : (lane >> 1), j = MX ? (lane & 3) : (lane & 1);
  const int bb = MX ? 17 : 9;
  uint8_t* dst = ws + blk * bb + 4 * j;
  if (!special && (MX ? e >= 1 : am <= 0x1p120f)) {
    float q[8];
    uint32_t w;
    if (MX) {
      // 1 / 2^(e-127) exactly (2^-127 is subnormal)
      const float r = e <= 253 ? __uint_as_float((254u - e) << 23) : __uint_as_float(0x00400000u);
      // products paired, "+ 0" scalar (see mx_encode_block)
      const float2 r2 = make_float2(r, r);
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        const float2 y = __fmul2_rn(make_float2(v[k], v[k + 1]), r2);
        q[k] = __fadd_rn(y.x, 0.0f);
        q[k + 1] = __fadd_rn(y.y, 0.0f);
      }
      w = fp4_word_signed(q, lut);
    } else {
      const NvScaleConst cst = g_nv_const[e];
      div_mk_n<8, false, true>(v, 0.0f, 0.0f, cst.scale, cst.rcp, q);
      w = fp4_word(q, v, -cst.t0, lut);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) dst[i] = (uint8_t)(w >> (8 * i));
  } else {
    float t[8];
    thr_load(&thr[e], t);
    if (!special) {
#pragma unroll
      for (int i = 0; i < 4; i++)
        dst[i] = (uint8_t)((fp4_encode_plain(v[2 * i], t) << 4) | fp4_encode_plain(v[2 * i + 1], t));
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++)
        dst[i] = (uint8_t)((fp4_encode(v[2 * i], t, z) << 4) | fp4_encode(v[2 * i + 1], t, z));
    }
  }
  if (j == (MX ? 3 : 1)) ws[blk * bb + bb - 1] = e;
}

// write a warp's staged bytes: whole 16-byte (NVFP4) / 8-byte (MXFP4) stores
// when the destination is aligned and the whole slice may be written, else
// bytes up to `limit`
template <bool MX>
__device__ __forceinline__ void flush_warp(const uint8_t* ws, uint8_t* dst, int64_t limit) {
  const int lane = threadIdx.x & 31;
  const int nbytes = MX ? kMxWarpBytes : kNvWarpBytes;
  const uintptr_t al = MX ? 7u : 15u;
  if (limit >= nbytes && ((reinterpret_cast<uintptr_t>(dst) & al) == 0)) {
    if (MX) {
      if (lane < nbytes / 8) reinterpret_cast<uint2*>(dst)[lane] = reinterpret_cast<const uint2*>(ws)[lane];
    } else {
      if (lane < nbytes / 16) reinterpret_cast<uint4*>(dst)[lane] = reinterpret_cast<const uint4*>(ws)[lane];
    }
  } else {
    const int m = (int)(limit < nbytes ? (limit > 0 ? limit : 0) : nbytes);
    for (int i = lane; i < m; i += 32) dst[i] = ws[i];
  }
}

__device__ __forceinline__ void store_elem8(int kind, const float v[8], uint8_t* dst) {
  if (kind == Q_FP16 || kind == Q_BF16) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint32_t lo = kind == Q_FP16 ? f32_to_f16_bits(v[2 * i]) : f32_to_bf16_bits(v[2 * i]);
      uint32_t hi = kind == Q_FP16 ? f32_to_f16_bits(v[2 * i + 1]) : f32_to_bf16_bits(v[2 * i + 1]);
      w[i] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    uint32_t w[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      uint32_t b = kind == Q_FP8_E5M2 ? f32_to_e5m2(v[i]) : f32_to_e4m3(v[i]);
      w[i >> 2] |= b << ((i & 3) * 8);
    }
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  }
}

// per-tensor scale from the amax slot (float bits; amax >= 0)
__device__ __forceinline__ float tensor_scale_from_amax(int kind, uint32_t amax_bits) {
  const float amax = __uint_as_float(amax_bits);
  float s = __fdiv_rn(amax, kind == Q_NVFP4_TENSOR ? 2688.0f : 448.0f);
  if (!(s > 0.0f) || s == __uint_as_float(0x7f800000u)) s = 1.0f;
  return s;
}

// NVFP4 with a per-tensor scale s_t encodes q = RN(x / s_t) against the
// block-scale thresholds Q = X_T(bs).  x -> RN(x / s_t) is monotone, so
// RN(|x| / s_t) >= Q exactly when |x| >= X'(Q), the least float whose IEEE
// quotient by s_t reaches Q; the block amax of q is RN(amax|x| / s_t) for the
// same reason.  A requant job therefore builds the composite table X'(X_T(bs))
// for s_t once (one exact double product per threshold) and then encodes
// the raw master with compares only, dividing once per block instead of once
// per element.
__device__ __forceinline__ float composite_threshold(float Q, float s) {
  // RN(y) >= Q exactly when y is at least the midpoint m between Q and its
  // predecessor (at a tie RN picks the even encoding: Q itself when Q's last
  // bit is 0, else the predecessor, and then y must exceed m).  With
  // y = x / s that is x >= m * s, a product exact in double (m has at most
  // 26 significant bits, s 24); the least such float is m * s rounded up.
  // Q = +Inf: RN overflows from 2^128 - 2^103 up (a tie rounded to Inf).
  if (!(Q > 0.0f)) return Q;  // NaN: "never"; 0: every x
  const uint32_t qb = __float_as_uint(Q);
  const double m = qb == 0x7f800000u ? 0x1p128 - 0x1p103
                                      : 0.5 * ((double)__uint_as_float(qb - 1u) + (double)Q);
  const double P = m * (double)s;
  float x = __double2float_ru(P);
  if ((qb & 1u) && (double)x == P) x = __uint_as_float(__float_as_uint(x) + 1u);
  return x;
}

__device__ __forceinline__ float block_amax_reduce(float v) {
  __shared__ float sm[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  }
  __syncthreads();
  return v;
}

// ---------------------------------------------------------------------------
// Passes 2+3: the apply kernel.  A persistent grid pulls jobs from a job
// list with an atomic ticket.  An update job runs the optimizer over one
// chunk (unscale, clip, SGD/Adam/AdamW, direct requant, per-tensor amax) and
// then counts itself done for its tensor; a requant job re-quantises one
// chunk of a per-tensor-scaled tensor once every update job of that tensor is
// done (the scale needs the whole tensor's amax).  The host orders the list
// so a tensor's requant jobs come a grid-width after its last update job,
// interleaved with the next tensor's update jobs: the ALU-heavy requant work
// overlaps the memory-bound update work instead of running as its own pass.
// A job only ever waits for jobs fetched before it, which are held by
// running CTAs, so the wait always ends; it is still bounded by
// %globaltimer and reports through Decision::err instead of hanging.
// ---------------------------------------------------------------------------
struct ApplyArgs {
  OptConsts oc;
  int use_scaler;
  const Chunk* chunks;  // update chunk table (requant jobs index it too)
  const uint32_t* jobs; // bit 31: requant job; low bits: chunk index
  int njobs;
  const TensorDesc* tensors;
  float* master;
  float* s1;
  float* s2;
  const void* grad;
  uint8_t* qout;
  uint32_t* amax_slots;
  float* qscale;
  uint32_t* sync;  // [0] job ticket, [1..] update jobs done per tensor
  Decision* dec;
  unsigned long long wait_ns;  // bound on a requant job's readiness wait (2 s unless a test shortens it)
};

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int GDT, int OPT>
__device__ __forceinline__ void update_chunk(const ApplyArgs& a, const Chunk& ch, const Divisor& dv, bool clipped,
                                             float coef, const Fp4Thr* s_mx, const Fp4Thr* s_nv, const uint8_t* s_lut,
                                             uint8_t* stage) {
  const OptConsts& oc = a.oc;
  const TensorDesc td = a.tensors[ch.tensor];
  const int kind = td.quant;
  const bool tensor_scaled = (kind == Q_FP8_E4M3_TENSOR || kind == Q_NVFP4_TENSOR);
  float amax = 0.0f;
  const int64_t end = ch.start + ch.len;
  for (int64_t tb = ch.start; tb < end; tb += kTile) {
    const int64_t e0 = tb + (int64_t)threadIdx.x * kVec;
    const bool act = e0 < end;
    float p[8], m[8], v[8], g[8];
    if (act) {
      const float4* pp = reinterpret_cast<const float4*>(a.master + e0);
      float4 p0 = __ldcs(pp), p1 = __ldcs(pp + 1);
      p[0] = p0.x; p[1] = p0.y; p[2] = p0.z; p[3] = p0.w;
      p[4] = p1.x; p[5] = p1.y; p[6] = p1.z; p[7] = p1.w;
      if (OPT != OPT_SGD || oc.use_mu) {
        const float4* mp = reinterpret_cast<const float4*>(a.s1 + e0);
        float4 m0 = __ldcs(mp), m1 = __ldcs(mp + 1);
        m[0] = m0.x; m[1] = m0.y; m[2] = m0.z; m[3] = m0.w;
        m[4] = m1.x; m[5] = m1.y; m[6] = m1.z; m[7] = m1.w;
      }
      if (OPT == OPT_ADAM || OPT == OPT_ADAMW || (OPT == OPT_RMSPROP && oc.use_mu)) {
        const float4* vp = reinterpret_cast<const float4*>(a.s2 + e0);
        float4 v0 = __ldcs(vp), v1 = __ldcs(vp + 1);
        v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
        v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
      }
      grad8<GDT>(a.grad, e0, a.use_scaler, dv, g);
#pragma unroll
      for (int k = 0; k < 8; k++) {
        float gk = clipped ? __fmul_rn(g[k], coef) : g[k];
        if (OPT == OPT_SGD)
          sgd_elem(p[k], gk, m[k], oc);
        else if (OPT == OPT_ADAM)
          adam_elem<false>(p[k], gk, m[k], v[k], oc);
        else if (OPT == OPT_ADAMW)
          adam_elem<true>(p[k], gk, m[k], v[k], oc);
        else if (OPT == OPT_LION)
          lion_elem(p[k], gk, m[k], oc);
        else if (OPT == OPT_RMSPROP)
          rmsprop_elem(p[k], gk, m[k], v[k], oc);
        else
          adagrad_elem(p[k], gk, m[k], oc);
      }
      float4* pw = reinterpret_cast<float4*>(a.master + e0);
      pw[0] = make_float4(p[0], p[1], p[2], p[3]);
      pw[1] = make_float4(p[4], p[5], p[6], p[7]);
      if (OPT != OPT_SGD || oc.use_mu) {
        float4* mw = reinterpret_cast<float4*>(a.s1 + e0);
        __stcs(mw, make_float4(m[0], m[1], m[2], m[3]));
        __stcs(mw + 1, make_float4(m[4], m[5], m[6], m[7]));
      }
      if (OPT == OPT_ADAM || OPT == OPT_ADAMW || (OPT == OPT_RMSPROP && oc.use_mu)) {
        float4* vw = reinterpret_cast<float4*>(a.s2 + e0);
        __stcs(vw, make_float4(v[0], v[1], v[2], v[3]));
        __stcs(vw + 1, make_float4(v[4], v[5], v[6], v[7]));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) p[k] = 0.0f;
    }
    // ---- requant epilogue (uniform per chunk) ----
    if (kind == Q_NONE) continue;
    if (tensor_scaled) {
#pragma unroll
      for (int k = 0; k < 8; k++) amax = amax_acc(amax, p[k]);
    } else if (kind == Q_MXFP4 || kind == Q_NVFP4) {
      // warp-uniform: the warp's first element is inside the chunk
      if (tb + (int64_t)(threadIdx.x & ~31) * kVec < end) {
        const int64_t tile_in_tensor = (tb - td.off) / kTile;
        const int w = threadIdx.x >> 5;
        uint8_t* ws = stage + w * kWarpStage;
        if (kind == Q_MXFP4) {
          stage_fp4<true>(p, ws, s_mx, s_lut);
          __syncwarp();
          flush_warp<true>(ws, a.qout + td.qoff + tile_in_tensor * kMxTileBytes + w * kMxWarpBytes, kMxWarpBytes);
        } else {
          stage_fp4<false>(p, ws, s_nv, s_lut);
          __syncwarp();
          flush_warp<false>(ws, a.qout + td.qoff + tile_in_tensor * kNvTileBytes + w * kNvWarpBytes, kNvWarpBytes);
        }
        __syncwarp();
      }
    } else if (act) {
      const int esz = (kind == Q_FP16 || kind == Q_BF16) ? 2 : 1;
      store_elem8(kind, p, a.qout + td.qoff + (e0 - td.off) * esz);
    }
  }
  if (tensor_scaled) {
    const float bm = block_amax_reduce(amax);
    if (threadIdx.x == 0) atomicMax(&a.amax_slots[ch.tensor], __float_as_uint(bm));
    // publish: every thread's stores of this chunk, then the done count
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(&a.sync[1 + ch.tensor], 1u);
  }
}

// A requant job: one chunk of a per-tensor-scaled tensor once all of the
// tensor's update jobs are done.  NVFP4: one thread per 16-element block
// (ody_fp4fast.cuh), a warp per 32 consecutive blocks; FP8-E4M3: 8
// elements per thread.  The CTA keeps the composite t0 table of the last
// tensor it re-quantised.
__device__ __forceinline__ void requant_chunk(const ApplyArgs& a, const Chunk& ch, const Fp4Thr* s_nv,
                                              float* s_t0, int* s_t0_tensor, const uint8_t* s_lut, uint8_t* stage) {
  const TensorDesc td = a.tensors[ch.tensor];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint32_t* done = &a.sync[1 + ch.tensor];
    int ok = 1;
    if (ld_acquire(done) < (uint32_t)td.nchunks) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire(done) < (uint32_t)td.nchunks) {
        if (globaltimer_ns() - t0 > a.wait_ns) {
          ok = 0;
          atomicOr(&a.dec->err, 1);
          break;
        }
        __nanosleep(256);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int kind = td.quant;
  const float s = tensor_scale_from_amax(kind, __ldcg(&a.amax_slots[ch.tensor]));
  const float r = __frcp_rn(s);
  if (ch.start == td.off && threadIdx.x == 0) a.qscale[ch.tensor] = s;
  const int64_t end = ch.start + ch.len;
  if (kind == Q_NVFP4_TENSOR) {
    if (*s_t0_tensor != ch.tensor) {
      // composite t0 of every E4M3 code for this tensor's scale (the sign rule)
      for (int i = threadIdx.x; i < 128; i += blockDim.x) s_t0[i] = composite_threshold(s_nv[i].t[0], s);
      __syncthreads();
      if (threadIdx.x == 0) *s_t0_tensor = ch.tensor;
    }
    const bool st_fast = s >= 0x1p-60f && s <= 0x1p60f;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ws = stage + w * kWarpStage;
    const int64_t nb = ch.len / 16;
    const int64_t blk0 = (ch.start - td.off) / 16;  // the chunk's first block within the tensor
    for (int64_t b0 = (int64_t)w * 32; b0 < nb; b0 += (kThreads / 32) * 32) {
      const int64_t b = b0 + lane;
      float v[16];
      if (b < nb) {
        const float4* pp = reinterpret_cast<const float4*>(a.master + ch.start + b * 16);
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float4 t = __ldcg(pp + k);
          v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 16; k++) v[k] = 0.0f;
      }
      uint32_t cw[2];
      const uint32_t sb = nv_encode_block<true>(v, s, r, st_fast, false, s_t0, g_nv_const, s_nv, s_lut, cw);
      stage_blocks<2>(ws, cw, sb);
      __syncwarp();
      flush_warp_bytes(ws, a.qout + td.qoff + (blk0 + b0) * 9, 32 * 9, (nb - b0) * 9);
      __syncwarp();
    }
    return;
  }
  // FP8-E4M3 with a per-tensor scale; the next tile's master values are
  // loaded before this tile is encoded
  float4 n0 = make_float4(0.f, 0.f, 0.f, 0.f), n1 = n0;
  {
    const int64_t e0 = ch.start + (int64_t)threadIdx.x * kVec;
    if (e0 < end) {
      const float4* pp = reinterpret_cast<const float4*>(a.master + e0);
      n0 = __ldcg(pp);
      n1 = __ldcg(pp + 1);
    }
  }
  for (int64_t tb = ch.start; tb < end; tb += kTile) {
    const int64_t e0 = tb + (int64_t)threadIdx.x * kVec;
    const bool act = e0 < end;
    float x[8];
    const float4 p0 = n0, p1 = n1;
    if (e0 + kTile < end) {
      const float4* pp = reinterpret_cast<const float4*>(a.master + e0 + kTile);
      n0 = __ldcg(pp);
      n1 = __ldcg(pp + 1);
    }
    if (act) {
      x[0] = p0.x; x[1] = p0.y; x[2] = p0.z; x[3] = p0.w;
      x[4] = p1.x; x[5] = p1.y; x[6] = p1.z; x[7] = p1.w;
#pragma unroll
      for (int k = 0; k < 8; k++) x[k] = div_by(x[k], s, r);
      store_elem8(Q_FP8_E4M3, x, a.qout + td.qoff + (e0 - td.off));
    }
  }
}

template <int GDT, int OPT>
__global__ void __launch_bounds__(kThreads, 4) apply_kernel(ApplyArgs a) {
  __shared__ Fp4Thr s_mx[256];
  __shared__ Fp4Thr s_nv[128];
  __shared__ __align__(16) uint8_t stage[(kThreads / 32) * kWarpStage];
  __shared__ float s_t0[128];
  __shared__ int s_t0_tensor;
  __shared__ uint8_t s_lut[2048];
  __shared__ uint32_t s_next;
  // prologue independent of the preceding stats/finalize grid
  load_thr_smem(s_mx, s_nv);
  load_ladder_signed(s_lut);
  // wait for the preceding grid (a no-op without a programmatic dependency)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const Decision* dec = a.dec;
  if (dec->skip) return;
  const Divisor dv = make_divisor(unscale_divisor<GDT>(dec->scale_used));
  const bool clipped = dec->clipped != 0;
  const float coef = dec->coef;
  if (threadIdx.x == 0) {
    s_next = atomicAdd(&a.sync[0], 1u);
    s_t0_tensor = -1;
  }
  __syncthreads();
  uint32_t j = s_next;
  while (j < (uint32_t)a.njobs) {
    uint32_t nxt = 0;
    if (threadIdx.x == 0) nxt = atomicAdd(&a.sync[0], 1u);  // next job, fetched early
    const uint32_t job = a.jobs[j];
    const Chunk ch = a.chunks[job & ~kRequantJob];
    if (job & kRequantJob)
      requant_chunk(a, ch, s_nv, s_t0, &s_t0_tensor, s_lut, stage);
    else
      update_chunk<GDT, OPT>(a, ch, dv, clipped, coef, s_mx, s_nv, s_lut, stage);
    __syncthreads();
    if (threadIdx.x == 0) s_next = nxt;
    __syncthreads();
    j = s_next;
  }
}

template <int GDT, int OPT>
static int grid_for_apply(int device) {
  int sms = 148, per = 4;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, apply_kernel<GDT, OPT>, kThreads, 0);
  if (per < 1) per = 1;
  return sms * per;
}

int apply_grid(int gdt, int opt, int device) {
#define ODY_G(G, O) \
  if (gdt == G && opt == O) return grid_for_apply<G, O>(device);
  ODY_G(DT_F32, OPT_SGD) ODY_G(DT_F32, OPT_ADAM) ODY_G(DT_F32, OPT_ADAMW)
  ODY_G(DT_F32, OPT_LION) ODY_G(DT_F32, OPT_RMSPROP) ODY_G(DT_F32, OPT_ADAGRAD)
  ODY_G(DT_F16, OPT_SGD) ODY_G(DT_F16, OPT_ADAM) ODY_G(DT_F16, OPT_ADAMW)
  ODY_G(DT_F16, OPT_LION) ODY_G(DT_F16, OPT_RMSPROP) ODY_G(DT_F16, OPT_ADAGRAD)
  ODY_G(DT_BF16, OPT_SGD) ODY_G(DT_BF16, OPT_ADAM) ODY_G(DT_BF16, OPT_ADAMW)
  ODY_G(DT_BF16, OPT_LION) ODY_G(DT_BF16, OPT_RMSPROP) ODY_G(DT_BF16, OPT_ADAGRAD)
#undef ODY_G
  return 148;
}

cudaError_t launch_apply(int gdt, int opt, const OptConsts& oc, int use_scaler, const Chunk* chunks,
                         const uint32_t* jobs, int njobs, const TensorDesc* tensors, float* master, float* s1,
                         float* s2, const void* grad, uint8_t* qout, uint32_t* amax_slots, float* qscale,
                         uint32_t* sync, Decision* dec, int grid, cudaStream_t st, unsigned long long wait_ns) {
  ApplyArgs a{oc, use_scaler, chunks, jobs, njobs, tensors, master, s1, s2, grad, qout, amax_slots, qscale, sync,
              dec, wait_ns};
  // programmatic dependent launch: the CTAs start while the stats (or
  // finalize) grid is still running and wait on it inside the kernel
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define ODY_L(G, O)                                  \
  if (gdt == G && opt == O) {                        \
    return cudaLaunchKernelEx(&cfg, apply_kernel<G, O>, a); \
  }
  ODY_L(DT_F32, OPT_SGD) ODY_L(DT_F32, OPT_ADAM) ODY_L(DT_F32, OPT_ADAMW)
  ODY_L(DT_F32, OPT_LION) ODY_L(DT_F32, OPT_RMSPROP) ODY_L(DT_F32, OPT_ADAGRAD)
  ODY_L(DT_F16, OPT_SGD) ODY_L(DT_F16, OPT_ADAM) ODY_L(DT_F16, OPT_ADAMW)
  ODY_L(DT_F16, OPT_LION) ODY_L(DT_F16, OPT_RMSPROP) ODY_L(DT_F16, OPT_ADAGRAD)
  ODY_L(DT_BF16, OPT_SGD) ODY_L(DT_BF16, OPT_ADAM) ODY_L(DT_BF16, OPT_ADAMW)
  ODY_L(DT_BF16, OPT_LION) ODY_L(DT_BF16, OPT_RMSPROP) ODY_L(DT_BF16, OPT_ADAGRAD)
#undef ODY_L
  return cudaErrorInvalidValue;
}

const void* apply_kernel_fn(int gdt, int opt) {
#define ODY_F(G, O) \
  if (gdt == G && opt == O) return reinterpret_cast<const void*>(&apply_kernel<G, O>);
  ODY_F(DT_F32, OPT_SGD) ODY_F(DT_F32, OPT_ADAM) ODY_F(DT_F32, OPT_ADAMW)
  ODY_F(DT_F32, OPT_LION) ODY_F(DT_F32, OPT_RMSPROP) ODY_F(DT_F32, OPT_ADAGRAD)
  ODY_F(DT_F16, OPT_SGD) ODY_F(DT_F16, OPT_ADAM) ODY_F(DT_F16, OPT_ADAMW)
  ODY_F(DT_F16, OPT_LION) ODY_F(DT_F16, OPT_RMSPROP) ODY_F(DT_F16, OPT_ADAGRAD)
  ODY_F(DT_BF16, OPT_SGD) ODY_F(DT_BF16, OPT_ADAM) ODY_F(DT_BF16, OPT_ADAMW)
  ODY_F(DT_BF16, OPT_LION) ODY_F(DT_BF16, OPT_RMSPROP) ODY_F(DT_BF16, OPT_ADAGRAD)
#undef ODY_F
  return nullptr;
}

cudaError_t set_apply_node(cudaGraphExec_t exec, cudaGraphNode_t node, int gdt, int opt, const OptConsts& oc,
                           int use_scaler, const Chunk* chunks, const uint32_t* jobs, int njobs,
                           const TensorDesc* tensors, float* master, float* s1, float* s2, const void* grad,
                           uint8_t* qout, uint32_t* amax_slots, float* qscale, uint32_t* sync, Decision* dec,
                           int grid, unsigned long long wait_ns) {
  ApplyArgs a{oc, use_scaler, chunks, jobs, njobs, tensors, master, s1, s2, grad, qout, amax_slots, qscale, sync,
              dec, wait_ns};
  void* args[1] = {&a};
  cudaKernelNodeParams kp = {};
  kp.func = const_cast<void*>(apply_kernel_fn(gdt, opt));
  if (!kp.func) return cudaErrorInvalidValue;
  kp.gridDim = dim3(grid);
  kp.blockDim = dim3(kThreads);
  kp.sharedMemBytes = 0;
  kp.kernelParams = args;
  kp.extra = nullptr;
  return cudaGraphExecKernelNodeSetParams(exec, node, &kp);
}

// ---------------------------------------------------------------------------
// Standalone quantise / dequantise of one tensor (AnyTensor.to_* / from_*,
// src/odyssey/tensor/tensor_dtype_conv.mojo:13-494).  Source float32 or
// bfloat16 (exact upcast first).  n is arbitrary; the last block is zero
// padded as in the reference (tensor_dtype_conv.mojo:306-307).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void load_src8(int sdt, const void* x, int64_t n, int64_t e0, float v[8]) {
  if (e0 + 8 <= n) {
    if (sdt == DT_F32) {
      const float* p = reinterpret_cast<const float*>(x) + e0;
      if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        float4 a = __ldcs(reinterpret_cast<const float4*>(p)), b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        return;
      }
    } else {
      const uint16_t* p = reinterpret_cast<const uint16_t*>(x) + e0;
      if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        uint4 r = __ldcs(reinterpret_cast<const uint4*>(p));
        uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = bf16_bits_to_f32((uint16_t)(w[k >> 1] >> ((k & 1) * 16)));
        return;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const int64_t i = e0 + k;
    float val = 0.0f;
    if (i < n)
      val = sdt == DT_F32 ? reinterpret_cast<const float*>(x)[i]
                          : bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(x)[i]);
    v[k] = val;
  }
}

// Per-tensor amax (NaN ignored, as the reference's compare) into out[0] and
// the smallest nonzero magnitude into out[1] (float bits; out[1] starts at
// 0xFFFFFFFF): one resident wave of CTAs, each thread with eight 16-byte
// loads in flight per round.
template <int SDT>
__global__ void __launch_bounds__(kThreads) amax_kernel(const void* x, int64_t n, uint32_t* out) {
  constexpr int EPV = SDT == DT_F32 ? 4 : 8;  // elements per 16-byte vector
  constexpr int U = 8;
  float am = 0.0f;
  uint32_t mn1 = 0xFFFFFFFFu;  // smallest (|v| bits - 1): zero wraps to the top, NaN sorts above +Inf
  auto acc = [&](float v) {
    am = fmaxf(am, fabsf(v));
    mn1 = min(mn1, (__float_as_uint(v) & 0x7FFFFFFFu) - 1u);
  };
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  const int64_t nv = aligned ? n / EPV : 0;  // whole vectors
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (U - 1) * stride < nv; i += U * stride) {
    uint4 r[U];
#pragma unroll
    for (int u = 0; u < U; u++) r[u] = __ldcg(xv + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        if (SDT == DT_F32) {
          acc(__uint_as_float(w[k]));
        } else {
          acc(__uint_as_float(w[k] << 16));
          acc(__uint_as_float(w[k] & 0xFFFF0000u));
        }
      }
    }
  }
  for (; i < nv; i += stride) {
    const uint4 r = __ldcg(xv + i);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      if (SDT == DT_F32) {
        acc(__uint_as_float(w[k]));
      } else {
        acc(__uint_as_float(w[k] << 16));
        acc(__uint_as_float(w[k] & 0xFFFF0000u));
      }
    }
  }
  // the ragged tail (or everything, for an unaligned source)
  for (int64_t e = nv * EPV + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
    const float v = SDT == DT_F32 ? reinterpret_cast<const float*>(x)[e]
                                  : bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(x)[e]);
    acc(v);
  }
  am = block_amax_reduce(am);
  // the smallest nonzero magnitude (bits; anything from +Inf up means none)
  uint32_t mn = mn1 >= 0x7F800000u ? 0x7F800000u : mn1 + 1u;
  mn = 0x7F800000u - __float_as_uint(block_amax_reduce(__uint_as_float(0x7F800000u - mn)));
  if (threadIdx.x == 0) {
    atomicMax(out, __float_as_uint(am));
    atomicMin(out + 1, mn);
  }
}

static int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

cudaError_t launch_amax(int sdt, const void* x, int64_t n, uint32_t* amax, cudaStream_t st) {
  static int per_sm[2] = {0, 0};
  const int t = sdt == DT_F32 ? 0 : 1;
  if (per_sm[t] == 0) {
    int k = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, sdt == DT_F32 ? amax_kernel<DT_F32> : amax_kernel<DT_BF16>,
                                                  kThreads, 0);
    per_sm[t] = k > 0 ? k : 1;
  }
  const int64_t want = (n / 8 + kThreads - 1) / kThreads + 1;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count() * per_sm[t]));
  if (sdt == DT_F32)
    amax_kernel<DT_F32><<<grid, kThreads, 0, st>>>(x, n, amax);
  else
    amax_kernel<DT_BF16><<<grid, kThreads, 0, st>>>(x, n, amax);
  return cudaGetLastError();
}

// FP16 / BF16 / FP8 kinds (with or without a per-tensor scale): 8 elements
// per thread, the next tile's values loaded before this tile is converted.
__global__ void __launch_bounds__(kThreads) quantize_kernel(int kind, int sdt, const void* x, int64_t n,
                                                            uint8_t* out, int64_t out_bytes,
                                                            const uint32_t* amax, float* tscale) {
  const bool scaled = kind == Q_FP8_E4M3_TENSOR;
  const float s = scaled ? tensor_scale_from_amax(kind, *amax) : 1.0f;
  const float r = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0 && tscale) *tscale = s;
  const int64_t ntiles = (n + kTile - 1) / kTile;
  float nx[8];
  if ((int64_t)blockIdx.x < ntiles) load_src8(sdt, x, n, (int64_t)blockIdx.x * kTile + (int64_t)threadIdx.x * kVec, nx);
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t e0 = t * kTile + (int64_t)threadIdx.x * kVec;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = nx[k];
    if (t + gridDim.x < ntiles) load_src8(sdt, x, n, e0 + (int64_t)gridDim.x * kTile, nx);
    if (scaled) {
#pragma unroll
      for (int k = 0; k < 8; k++) v[k] = div_by(v[k], s, r);
    }
    const int esz = (kind == Q_FP16 || kind == Q_BF16) ? 2 : 1;
    const int qk = scaled ? Q_FP8_E4M3 : kind;
    uint8_t* dst = out + e0 * esz;
    if (e0 + 8 <= n && (reinterpret_cast<uintptr_t>(dst) & (esz == 2 ? 15u : 7u)) == 0) {
      store_elem8(qk, v, dst);
    } else {
      for (int k = 0; k < 8 && e0 + k < n; k++) {
        if (esz == 2) {
          uint16_t h = qk == Q_FP16 ? f32_to_f16_bits(v[k]) : f32_to_bf16_bits(v[k]);
          reinterpret_cast<uint16_t*>(out)[e0 + k] = h;
        } else {
          out[e0 + k] = qk == Q_FP8_E5M2 ? f32_to_e5m2(v[k]) : f32_to_e4m3(v[k]);
        }
      }
    }
  }
  (void)out_bytes;
}

// ---------------------------------------------------------------------------
// FP4 kinds: one thread per block (16 elements for NVFP4, 32 for MXFP4),
// encoded with the cheap exact path of ody_fp4fast.cuh.  A warp covers 32
// consecutive blocks, whose 288 (NVFP4) or 544 (MXFP4) output bytes it
// stages in shared memory and writes with 16-byte stores.
// ---------------------------------------------------------------------------
template <int SDT, int NE>
__device__ __forceinline__ void load_block(const void* x, int64_t n, int64_t e0, float* v) {
#pragma unroll
  for (int k = 0; k < NE; k += 8) load_src8(SDT, x, n, e0 + k, v + k);
}

template <int KIND, int SDT>
__global__ void __launch_bounds__(kThreads) quant_fp4_kernel(const void* x, int64_t n, uint8_t* out,
                                                             int64_t out_bytes, const uint32_t* amax,
                                                             float* tscale) {
  constexpr bool MX = KIND == Q_MXFP4 || KIND == Q_MXFP4_OCP;
  constexpr bool TS = KIND == Q_NVFP4_TENSOR;
  constexpr int BE = MX ? 32 : 16;  // elements per block
  constexpr int BB = MX ? 17 : 9;   // bytes per block
  constexpr int WB = 32 * BB;       // bytes per warp
  __shared__ __align__(16) uint8_t stage[kThreads / 32][WB];
  __shared__ float s_t0[TS ? 128 : 1];
  __shared__ uint8_t s_lut[2048];
  load_ladder_signed(s_lut);
  __syncthreads();
  float st = 1.0f, rst = 1.0f;
  bool st_fast = true, sign_fast = false;
  if (TS) {
    st = tensor_scale_from_amax(KIND, *amax);
    rst = __frcp_rn(st);
    st_fast = st >= 0x1p-60f && st <= 0x1p60f;
    // amax[1]: the smallest nonzero magnitude (all ones: none)
    const float mnz = __uint_as_float(amax[1]);
    sign_fast = st_fast && !(mnz < __fmul_rn(st, 0x1p-113f));
    for (int i = threadIdx.x; i < 128; i += blockDim.x) s_t0[i] = composite_threshold(g_thr_nv[i].t[0], st);
    __syncthreads();
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && tscale) *tscale = st;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ws = stage[w];
  const int64_t nblocks = (n + BE - 1) / BE;
  const int64_t step = (int64_t)gridDim.x * (kThreads / 32) * 32;
  for (int64_t b0 = ((int64_t)blockIdx.x * (kThreads / 32) + w) * 32; b0 < nblocks; b0 += step) {
    const int64_t b = b0 + lane;
    float v[BE];
    load_block<SDT, BE>(x, n, b * BE, v);  // zero beyond n
    uint32_t cw[BE / 8];
    uint32_t sb;
    if (MX)
      sb = KIND == Q_MXFP4_OCP ? mx_ocp_encode_block(v, cw) : mx_encode_block(v, g_thr_mx, s_lut, cw);
    else
      sb = nv_encode_block<TS>(v, st, rst, st_fast, sign_fast, s_t0, g_nv_const, g_thr_nv, s_lut, cw);
    stage_blocks<BE / 8>(ws, cw, sb);
    __syncwarp();
    flush_warp_bytes(ws, out + b0 * BB, WB, out_bytes - b0 * BB);
    __syncwarp();
  }
}

// The same with the input staged through shared memory: each warp fills a
// ring of two or three segments (32 blocks each) with coalesced 16-byte
// cp.async copies, several segments ahead of the one it encodes, so that the
// loads of a thread are neither strided nor waited for one block at a time.
// Needs a 16-byte-aligned source.
// stages per warp ring: three, or two where a segment is 4 KB (MXFP4 from
// float32), which keeps three CTAs per SM
template <int SEGB>
struct Fp4Stages {
  static constexpr int N = SEGB >= 4096 ? 2 : 3;
};

template <int KIND, int SDT>
struct Fp4Pipe {
  static constexpr int BE = (KIND == Q_MXFP4 || KIND == Q_MXFP4_OCP) ? 32 : 16;
  static constexpr int BB = (KIND == Q_MXFP4 || KIND == Q_MXFP4_OCP) ? 17 : 9;
  static constexpr int ESZ = SDT == DT_F32 ? 4 : 2;
  static constexpr int P = BE * ESZ / 16;  // 16-byte slots per block
  static constexpr int SEG = 32 * P * 16;  // input bytes per warp segment
  static constexpr int WB = (32 * BB + 15) / 16 * 16;
  static constexpr int NS = Fp4Stages<SEG>::N;
  static constexpr int SMEM = (kThreads / 32) * (NS * SEG + WB);
};

template <int KIND, int SDT>
__global__ void __launch_bounds__(kThreads) quant_fp4_pipe_kernel(const void* x, int64_t n, uint8_t* out,
                                                                  int64_t out_bytes, const uint32_t* amax,
                                                                  float* tscale) {
  using PP = Fp4Pipe<KIND, SDT>;
  constexpr bool MX = KIND == Q_MXFP4 || KIND == Q_MXFP4_OCP;
  constexpr bool TS = KIND == Q_NVFP4_TENSOR;
  constexpr int NS = PP::NS;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ float s_t0[TS ? 128 : 1];
  __shared__ uint8_t s_lut[2048];
  load_ladder_signed(s_lut);
  __syncthreads();
  float st = 1.0f, rst = 1.0f;
  bool st_fast = true, sign_fast = false;
  if (TS) {
    st = tensor_scale_from_amax(KIND, *amax);
    rst = __frcp_rn(st);
    st_fast = st >= 0x1p-60f && st <= 0x1p60f;
    // amax[1]: the smallest nonzero magnitude (all ones: none)
    const float mnz = __uint_as_float(amax[1]);
    sign_fast = st_fast && !(mnz < __fmul_rn(st, 0x1p-113f));
    for (int i = threadIdx.x; i < 128; i += blockDim.x) s_t0[i] = composite_threshold(g_thr_nv[i].t[0], st);
    __syncthreads();
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && tscale) *tscale = st;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = dsm + w * (NS * PP::SEG);
  uint8_t* ws = dsm + (kThreads / 32) * (NS * PP::SEG) + w * PP::WB;
  const int64_t in_bytes = n * PP::ESZ;
  const int64_t ngroups = ((n + PP::BE - 1) / PP::BE + 31) / 32;
  const int64_t gstep = (int64_t)gridDim.x * (kThreads / 32);
  const int64_t g0 = (int64_t)blockIdx.x * (kThreads / 32) + w;
  const char* src = reinterpret_cast<const char*>(x);
  constexpr int OP = (32 * PP::BB + 15) / 16;  // 16-byte output pieces per warp
  const bool out_al = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  // loop-invariant swizzled offsets of this lane's fill and read slots
  uint32_t fill_at[PP::P], read_at[PP::P];
  const uint32_t ring_s = smem_u32(ring);
#pragma unroll
  for (int k = 0; k < PP::P; k++) {
    fill_at[k] = ring_s + swz16(k * 32 + lane) * 16;
    read_at[k] = swz16(lane * PP::P + k) * 16;
  }
  auto issue = [&](int64_t g, int s) {
    const int64_t off = g * PP::SEG;
    if (off + PP::SEG <= in_bytes) {
      const char* b = src + off + 16 * lane;
#pragma unroll
      for (int k = 0; k < PP::P; k++) cp_async16(fill_at[k] + s * PP::SEG, b + 512 * k, 16);
    } else {
#pragma unroll
      for (int k = 0; k < PP::P; k++) {
        const int64_t o = off + 512 * k + 16 * lane;
        const int64_t rem = in_bytes - o;
        const int bytes = rem >= 16 ? 16 : (rem > 0 ? (int)rem : 0);
        cp_async16(fill_at[k] + s * PP::SEG, bytes > 0 ? src + o : src, bytes);
      }
    }
  };
#pragma unroll
  for (int s = 0; s < NS - 1; s++) {
    const int64_t g = g0 + s * gstep;
    if (g < ngroups) issue(g, s);
    cp_async_commit();
  }
  int64_t g = g0;
  while (g < ngroups) {
#pragma unroll
    for (int s = 0; s < NS; s++) {  // this iteration encodes stage s (compile-time)
      if (g >= ngroups) break;
      const int64_t gn = g + (NS - 1) * gstep;
      if (gn < ngroups) issue(gn, (s + NS - 1) % NS);
      cp_async_commit();
      cp_async_wait<NS - 1>();
      __syncwarp();
      float v[PP::BE];
      const uint8_t* seg = ring + s * PP::SEG;
#pragma unroll
      for (int j = 0; j < PP::P; j++) {
        const uint4 r = *reinterpret_cast<const uint4*>(seg + read_at[j]);
        if (SDT == DT_F32) {
          v[4 * j] = __uint_as_float(r.x);
          v[4 * j + 1] = __uint_as_float(r.y);
          v[4 * j + 2] = __uint_as_float(r.z);
          v[4 * j + 3] = __uint_as_float(r.w);
        } else {
          const uint32_t ww[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            v[8 * j + 2 * k] = __uint_as_float(ww[k] << 16);
            v[8 * j + 2 * k + 1] = __uint_as_float(ww[k] & 0xFFFF0000u);
          }
        }
      }
      __syncwarp();  // every lane has its block: the slot may be refilled
      uint32_t cw[PP::BE / 8];
      uint32_t sb;
      if (MX)
        sb = KIND == Q_MXFP4_OCP ? mx_ocp_encode_block(v, cw) : mx_encode_block(v, g_thr_mx, s_lut, cw);
      else
        sb = nv_encode_block<TS>(v, st, rst, st_fast, sign_fast, s_t0, g_nv_const, g_thr_nv, s_lut, cw);
      stage_blocks<PP::BE / 8>(ws, cw, sb);
      __syncwarp();
      const int64_t ob = g * 32 * PP::BB;
      if (out_al && ob + 32 * PP::BB <= out_bytes) {
        uint4* dst = reinterpret_cast<uint4*>(out + ob);
#pragma unroll
        for (int i = 0; i < (OP + 31) / 32; i++)
          if (i * 32 + lane < OP) dst[i * 32 + lane] = reinterpret_cast<const uint4*>(ws)[i * 32 + lane];
      } else {
        flush_warp_bytes(ws, out + ob, 32 * PP::BB, out_bytes - ob);
      }
      __syncwarp();
      g += gstep;
    }
  }
  cp_async_wait<0>();
}

template <int KIND, int SDT>
static cudaError_t launch_fp4_pipe(const void* x, int64_t n, uint8_t* out, int64_t out_bytes, const uint32_t* amax,
                                   float* tscale, cudaStream_t st) {
  using PP = Fp4Pipe<KIND, SDT>;
  static int per_sm[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  auto fn = quant_fp4_pipe_kernel<KIND, SDT>;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (per_sm[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, PP::SMEM);
    if (e != cudaSuccess) return e;
    int k = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, fn, kThreads, PP::SMEM);
    if (e != cudaSuccess) return e;
    per_sm[dev] = k > 0 ? k : 1;
  }
  const int64_t groups = ((n + PP::BE - 1) / PP::BE + 31) / 32;
  const int64_t want = (groups + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t cap = (int64_t)sm_count() * per_sm[dev];
  const int grid = (int)std::max<int64_t>(1, std::min(want, cap));
  fn<<<grid, kThreads, PP::SMEM, st>>>(x, n, out, out_bytes, amax, tscale);
  return cudaGetLastError();
}

template <int KIND>
static void launch_fp4_kind(int sdt, const void* x, int64_t n, uint8_t* out, int64_t out_bytes, const uint32_t* amax,
                            float* tscale, int grid, cudaStream_t st) {
  if (sdt == DT_F32)
    quant_fp4_kernel<KIND, DT_F32><<<grid, kThreads, 0, st>>>(x, n, out, out_bytes, amax, tscale);
  else
    quant_fp4_kernel<KIND, DT_BF16><<<grid, kThreads, 0, st>>>(x, n, out, out_bytes, amax, tscale);
}

static int64_t quant_bytes_dev(int kind, int64_t n) {
  switch (kind) {
    case Q_FP16:
    case Q_BF16:
      return 2 * n;
    case Q_FP8_E4M3:
    case Q_FP8_E5M2:
    case Q_FP8_E4M3_TENSOR:
      return n;
    case Q_MXFP4:
    case Q_MXFP4_OCP:
      return ((n + 31) / 32) * 17;
    case Q_NVFP4:
    case Q_NVFP4_TENSOR:
      return ((n + 15) / 16) * 9;
  }
  return 0;
}

cudaError_t launch_quantize(int kind, int sdt, const void* x, int64_t n, uint8_t* out,
                            const uint32_t* amax, float* tscale, cudaStream_t st) {
  if (kind == Q_MXFP4 || kind == Q_MXFP4_OCP || kind == Q_NVFP4 || kind == Q_NVFP4_TENSOR) {
    const int64_t be = (kind == Q_MXFP4 || kind == Q_MXFP4_OCP) ? 32 : 16;
    const int64_t warps = ((n + be - 1) / be + 31) / 32;
    const int64_t want = (warps + kThreads / 32 - 1) / (kThreads / 32);
    const int64_t cap = (int64_t)sm_count() * 4;
    const int grid = (int)std::max<int64_t>(1, std::min(want, cap));
    const int64_t ob = quant_bytes_dev(kind, n);
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
#define ODY_P(K)                                                                          \
  if (kind == K)                                                                          \
    return sdt == DT_F32 ? launch_fp4_pipe<K, DT_F32>(x, n, out, ob, amax, tscale, st)    \
                         : launch_fp4_pipe<K, DT_BF16>(x, n, out, ob, amax, tscale, st);
      ODY_P(Q_MXFP4) ODY_P(Q_MXFP4_OCP) ODY_P(Q_NVFP4) ODY_P(Q_NVFP4_TENSOR)
#undef ODY_P
    }
    if (kind == Q_MXFP4)
      launch_fp4_kind<Q_MXFP4>(sdt, x, n, out, ob, amax, tscale, grid, st);
    else if (kind == Q_MXFP4_OCP)
      launch_fp4_kind<Q_MXFP4_OCP>(sdt, x, n, out, ob, amax, tscale, grid, st);
    else if (kind == Q_NVFP4)
      launch_fp4_kind<Q_NVFP4>(sdt, x, n, out, ob, amax, tscale, grid, st);
    else
      launch_fp4_kind<Q_NVFP4_TENSOR>(sdt, x, n, out, ob, amax, tscale, grid, st);
    return cudaGetLastError();
  }
  int64_t ntiles = (n + kTile - 1) / kTile;
  int64_t cap = (int64_t)sm_count() * 8;
  int grid = (int)(ntiles < cap ? ntiles : cap);
  if (grid < 1) grid = 1;
  quantize_kernel<<<grid, kThreads, 0, st>>>(kind, sdt, x, n, out, quant_bytes_dev(kind, n), amax,
                                             tscale);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(kThreads) dequantize_kernel(int kind, const uint8_t* q, int64_t n,
                                                              int64_t qbytes, const float* tscale,
                                                              float* out) {
  __shared__ __align__(16) uint8_t stage[kNvTileBytes];
  const float ts = tscale ? *tscale : 1.0f;
  const bool scaled = (kind == Q_NVFP4_TENSOR || kind == Q_FP8_E4M3_TENSOR);
  const int64_t ntiles = (n + kTile - 1) / kTile;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t e0 = t * kTile + (int64_t)threadIdx.x * kVec;
    float v[8];
    const bool mx = kind == Q_MXFP4 || kind == Q_MXFP4_OCP;
    if (mx || kind == Q_NVFP4 || kind == Q_NVFP4_TENSOR) {
      const int tb = mx ? kMxTileBytes : kNvTileBytes;
      const int64_t off = t * tb;
      const int64_t lim = qbytes - off < tb ? qbytes - off : tb;
      for (int i = threadIdx.x; i < lim; i += blockDim.x) stage[i] = q[off + i];
      __syncthreads();
      if (kind == Q_MXFP4_OCP) {
        // OCP MX decode: the E2M1 value (0.5 included) times 2^(byte - 127); 0xFF is NaN
        const int blk = threadIdx.x >> 2, j = threadIdx.x & 3;
        const uint8_t sbyte = (blk * 17 + 16 < lim) ? stage[blk * 17 + 16] : 127;
        const float sf = sbyte == 0xFF ? __uint_as_float(0x7fc00000u)
                                       : (sbyte >= 1 ? __uint_as_float((uint32_t)sbyte << 23)
                                                     : __uint_as_float(0x00400000u));
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint8_t b = (blk * 17 + 4 * j + i < lim) ? stage[blk * 17 + 4 * j + i] : 0;
          v[2 * i] = e2m1_ocp_decode(b >> 4, sf);
          v[2 * i + 1] = e2m1_ocp_decode(b & 15, sf);
        }
      } else if (kind == Q_MXFP4) {
        const int blk = threadIdx.x >> 2, j = threadIdx.x & 3;
        const float sf = (blk * 17 + 16 < lim) ? e8m0_to_f32(stage[blk * 17 + 16]) : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint8_t b = (blk * 17 + 4 * j + i < lim) ? stage[blk * 17 + 4 * j + i] : 0;
          v[2 * i] = fp4_decode(b >> 4, sf);
          v[2 * i + 1] = fp4_decode(b & 15, sf);
        }
      } else {
        const int blk = threadIdx.x >> 1, j = threadIdx.x & 1;
        const float sf = (blk * 9 + 8 < lim) ? e4m3_to_f32(stage[blk * 9 + 8]) : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint8_t b = (blk * 9 + 4 * j + i < lim) ? stage[blk * 9 + 4 * j + i] : 0;
          v[2 * i] = fp4_decode(b >> 4, sf);
          v[2 * i + 1] = fp4_decode(b & 15, sf);
        }
      }
      __syncthreads();
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int64_t i = e0 + k;
        float val = 0.0f;
        if (i < n) {
          if (kind == Q_FP16)
            val = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(q)[i]);
          else if (kind == Q_BF16)
            val = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(q)[i]);
          else if (kind == Q_FP8_E5M2)
            val = e5m2_to_f32(q[i]);
          else
            val = e4m3_to_f32(q[i]);
        }
        v[k] = val;
      }
    }
    if (scaled) {
#pragma unroll
      for (int k = 0; k < 8; k++) v[k] = __fmul_rn(v[k], ts);
    }
    float* dst = out + e0;
    if (e0 + 8 <= n && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      __stcs(reinterpret_cast<float4*>(dst), make_float4(v[0], v[1], v[2], v[3]));
      __stcs(reinterpret_cast<float4*>(dst) + 1, make_float4(v[4], v[5], v[6], v[7]));
    } else {
      for (int k = 0; k < 8 && e0 + k < n; k++) dst[k] = v[k];
    }
  }
}

cudaError_t launch_dequantize(int kind, const uint8_t* q, int64_t n, const float* tscale, float* out,
                              cudaStream_t st) {
  int64_t ntiles = (n + kTile - 1) / kTile;
  int64_t cap = (int64_t)sm_count() * 6;
  int grid = (int)(ntiles < cap ? ntiles : cap);
  if (grid < 1) grid = 1;
  dequantize_kernel<<<grid, kThreads, 0, st>>>(kind, q, n, quant_bytes_dev(kind, n), tscale, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Single-op kernels (the reference's separate API functions).
// ---------------------------------------------------------------------------
__global__ void unscale_kernel(int dt, const void* g, int64_t n, float scale, void* out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (dt == DT_F32) {
      reinterpret_cast<float*>(out)[i] = __fdiv_rn(reinterpret_cast<const float*>(g)[i], scale);
    } else if (dt == DT_F16) {
      const float d = unscale_divisor<DT_F16>(scale);
      float x = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(g)[i]);
      reinterpret_cast<uint16_t*>(out)[i] = f32_to_f16_bits(__fdiv_rn(x, d));
    } else {
      const float d = unscale_divisor<DT_BF16>(scale);
      float x = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(g)[i]);
      reinterpret_cast<uint16_t*>(out)[i] = f32_to_bf16_bits(__fdiv_rn(x, d));
    }
  }
}

static int grid_for(int64_t n) {
  int64_t want = (n + kThreads - 1) / kThreads;
  int64_t cap = (int64_t)sm_count() * 8;
  int g = (int)(want < cap ? want : cap);
  return g < 1 ? 1 : g;
}

cudaError_t launch_unscale(int dt, const void* g, int64_t n, float scale, void* out, cudaStream_t st) {
  unscale_kernel<<<grid_for(n), kThreads, 0, st>>>(dt, g, n, scale, out);
  return cudaGetLastError();
}

__global__ void nonfinite_kernel(int dt, const void* g, int64_t n, unsigned long long* count) {
  long long c = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float x = dt == DT_F32 ? reinterpret_cast<const float*>(g)[i]
              : dt == DT_F16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t*>(g)[i])
                             : bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(g)[i]);
    c += !is_finite_f(x);
  }
  c = warp_sum(c);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(count, (unsigned long long)c);
}

cudaError_t launch_count_nonfinite(int dt, const void* g, int64_t n, unsigned long long* count,
                                   cudaStream_t st) {
  nonfinite_kernel<<<grid_for(n), kThreads, 0, st>>>(dt, g, n, count);
  return cudaGetLastError();
}

// sum of float32 squares in float64 (8-element float32 groups, as sq8),
// per-CTA partials + fixed-order final sum
// SQ64: squares taken in float64 (optimizer_utils.mojo:189-229); else float32
// squares reduced per 8 lanes (gradient_clipping.mojo:52-67,
// numerical_safety.mojo:581-594)
template <bool SQ64>
__global__ void sumsq_kernel(const float* g, int64_t n, StatsPartial* partials, unsigned* ticket,
                             double* total) {
  double acc = 0.0;
  long long dummy = 0;
  const int64_t ngroups = (n + 7) / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < ngroups; i += stride) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = (i * 8 + k < n) ? g[i * 8 + k] : 0.0f;
    if (SQ64) {
#pragma unroll
      for (int k = 0; k < 8; k++) acc = __dadd_rn(acc, __dmul_rn((double)v[k], (double)v[k]));
    } else {
      acc += (double)sq8(v);
    }
  }
  block_sum2(acc, dummy);
  __shared__ bool last;
  if (threadIdx.x == 0) {
    partials[blockIdx.x].sumsq = acc;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  double s = 0.0;
  long long c = 0;
  for (int j = threadIdx.x; j < (int)gridDim.x; j += blockDim.x) s += __ldcg(&partials[j].sumsq);
  block_sum2(s, c);
  if (threadIdx.x == 0) {
    *total += s;  // accumulated over the tensors of one call, in call order
    *ticket = 0u;
  }
}

cudaError_t launch_sumsq(const float* g, int64_t n, StatsPartial* partials, int grid, unsigned* ticket,
                         double* total, cudaStream_t st) {
  sumsq_kernel<false><<<grid, kThreads, 0, st>>>(g, n, partials, ticket, total);
  return cudaGetLastError();
}

cudaError_t launch_sumsq64(const float* g, int64_t n, StatsPartial* partials, int grid, unsigned* ticket,
                           double* total, cudaStream_t st) {
  sumsq_kernel<true><<<grid, kThreads, 0, st>>>(g, n, partials, ticket, total);
  return cudaGetLastError();
}

// clip_grad_global_norm_ (numerical_safety.mojo:760-815, mode 0) and
// clip_global_norm (optimizer_utils.mojo:303-348, mode 1): norm =
// sqrt(sumsq) in float64; when norm > max_norm and norm > 0 the factor is
// max_norm / norm in float64, applied as a float32 multiplier (mode 0) or as
// a float64 product rounded back to float32 (mode 1); coef[1] = 1 marks "scale"
__global__ void clip_variant_coef_kernel(const double* total, double max_norm, double* norm_out, double* coef) {
  const double norm = __dsqrt_rn(*total);
  *norm_out = norm;
  const bool clip = norm > max_norm && norm > 0.0;
  coef[0] = clip ? __ddiv_rn(max_norm, norm) : 1.0;
  coef[1] = clip ? 1.0 : 0.0;
}

__global__ void clip_variant_scale_kernel(float* g, int64_t n, const double* coef, int mode) {
  if (coef[1] == 0.0) return;
  const double c = coef[0];
  const float c32 = __double2float_rn(c);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    g[i] = mode == 0 ? __fmul_rn(g[i], c32) : __double2float_rn(__dmul_rn((double)g[i], c));
}

cudaError_t launch_clip_variant_coef(const double* total, double max_norm, double* norm_out, double* coef,
                                     cudaStream_t st) {
  clip_variant_coef_kernel<<<1, 1, 0, st>>>(total, max_norm, norm_out, coef);
  return cudaGetLastError();
}

cudaError_t launch_clip_variant_scale(float* g, int64_t n, const double* coef, int mode, cudaStream_t st) {
  clip_variant_scale_kernel<<<grid_for(n), kThreads, 0, st>>>(g, n, coef, mode);
  return cudaGetLastError();
}

// clip_gradients_by_global_norm (gradient_clipping.mojo:310-352)
__global__ void clip_coef_kernel(const double* total, float max_norm, float* norm_out, float* coef_out) {
  const float norm = __double2float_rn(__dsqrt_rn(*total));
  *norm_out = norm;
  *coef_out = norm > max_norm
                  ? __double2float_rn(__ddiv_rn((double)max_norm, __dadd_rn((double)norm, 1e-6)))
                  : 1.0f;
}

cudaError_t launch_clip_coef(const double* total, float max_norm, float* norm_out, float* coef_out,
                             cudaStream_t st) {
  clip_coef_kernel<<<1, 1, 0, st>>>(total, max_norm, norm_out, coef_out);
  return cudaGetLastError();
}

__global__ void scale_kernel(float* g, int64_t n, const float* coef) {
  const float c = *coef;
  if (c == 1.0f) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    g[i] = __fmul_rn(g[i], c);
}

cudaError_t launch_scale_inplace(float* g, int64_t n, const float* coef, cudaStream_t st) {
  scale_kernel<<<grid_for(n), kThreads, 0, st>>>(g, n, coef);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// FP4 singles: one value with its own power-of-two scale
// (MXFP4/NVFP4.from_float32 / from_float32_stochastic / to_float32,
// src/odyssey/core/types/mxfp4.mojo:303-491, nvfp4.mojo:290-481).
// ---------------------------------------------------------------------------
// _fp4_from_float32 (mxfp4.mojo:144-224) on RN(x / scale)
__device__ __forceinline__ uint8_t fp4_ladder_code(float x, float scale) {
  if (x != x) return 0x7;
  if (fabsf(x) == __uint_as_float(0x7f800000u)) return x > 0.0f ? 0x7 : 0xf;
  const float q = __fdiv_rn(x, scale);
  if (q == 0.0f) return 0;
  const uint8_t sign = q < 0.0f;
  const float a = fabsf(q);
  if (a >= 6.0f) return (uint8_t)((sign << 3) | 0x7);
  if (a < 0.5f) return (uint8_t)(sign << 3);
  const uint8_t code = a < 1.25f ? 0x2 : a < 1.75f ? 0x3 : a < 2.5f ? 0x4 : a < 3.5f ? 0x5 : a < 5.0f ? 0x6 : 0x7;
  return (uint8_t)((sign << 3) | code);
}

// _fp4_stochastic_round (mxfp4.mojo:398-483): the E2M1 bucket of |x/scale|,
// P(upper) = (|x/scale| - lower) / (upper - lower), one 32-bit LCG step of
// the seed, (state >> 8) / 2^24 < P picks the upper value
__device__ __forceinline__ uint8_t fp4_stochastic_code(float x, float scale, uint64_t seed) {
  const float q = __fdiv_rn(x, scale);
  const uint8_t sign = q < 0.0f;
  const float a = sign ? -q : q;
  float lo, hi;
  uint8_t lb, ub;
  if (a < 0.5f) return (uint8_t)(sign << 3);
  if (a < 1.0f) { lo = 0.0f; hi = 1.0f; lb = 0x0; ub = 0x2; }
  else if (a < 1.5f) { lo = 1.0f; hi = 1.5f; lb = 0x2; ub = 0x3; }
  else if (a < 2.0f) { lo = 1.5f; hi = 2.0f; lb = 0x3; ub = 0x4; }
  else if (a < 3.0f) { lo = 2.0f; hi = 3.0f; lb = 0x4; ub = 0x5; }
  else if (a < 4.0f) { lo = 3.0f; hi = 4.0f; lb = 0x5; ub = 0x6; }
  else if (a < 6.0f) { lo = 4.0f; hi = 6.0f; lb = 0x6; ub = 0x7; }
  else return (uint8_t)((sign << 3) | 0x7);
  const float p_up = __fdiv_rn(__fsub_rn(a, lo), __fsub_rn(hi, lo));
  const uint32_t st = 1103515245u * (uint32_t)seed + 12345u;
  const float r = __fdiv_rn((float)(st >> 8), 16777216.0f);
  return (uint8_t)((sign << 3) | (r < p_up ? ub : lb));
}

__global__ void fp4_single_encode_kernel(int mx, const float* x, int64_t n, const uint64_t* seeds, uint8_t* vals,
                                         uint8_t* scs) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    const uint8_t unit = mx ? 127 : 0x3C;
    if (v != v || fabsf(v) == __uint_as_float(0x7f800000u)) {
      vals[i] = fp4_ladder_code(v, 1.0f);
      scs[i] = unit;
      continue;
    }
    if (v == 0.0f) {
      vals[i] = 0;
      scs[i] = unit;
      continue;
    }
    const float ax = v > 0.0f ? v : -v;
    float sv = 1.0f;
    int ev = 0;
    // at most 128 doublings (sv reaches Inf, the quotient 0) and 127 halvings
    while (__fdiv_rn(ax, sv) > 6.0f) {
      sv = __fmul_rn(sv, 2.0f);
      ev++;
    }
    while (__fdiv_rn(ax, sv) < 0.5f && ev > (mx ? -127 : -7)) {
      sv = __fdiv_rn(sv, 2.0f);
      ev--;
    }
    const uint8_t e = mx ? e8m0_from_f32(sv) : e4m3_scale_from_f32(sv);
    const float sf = mx ? e8m0_to_f32(e) : e4m3_to_f32(e);
    scs[i] = e;
    vals[i] = seeds ? fp4_stochastic_code(v, sf, seeds[i]) : fp4_ladder_code(v, sf);
  }
}

__global__ void fp4_single_decode_kernel(int mx, const uint8_t* vals, const uint8_t* scs, int64_t n, float* out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float sf = mx ? e8m0_to_f32(scs[i]) : e4m3_to_f32(scs[i]);
    out[i] = fp4_decode(vals[i] & 0xfu, sf);
  }
}

cudaError_t launch_fp4_single_encode(int mx, const float* x, int64_t n, const uint64_t* seeds, uint8_t* vals,
                                     uint8_t* scs, cudaStream_t st) {
  fp4_single_encode_kernel<<<grid_for(n), kThreads, 0, st>>>(mx, x, n, seeds, vals, scs);
  return cudaGetLastError();
}

cudaError_t launch_fp4_single_decode(int mx, const uint8_t* vals, const uint8_t* scs, int64_t n, float* out,
                                     cudaStream_t st) {
  fp4_single_decode_kernel<<<grid_for(n), kThreads, 0, st>>>(mx, vals, scs, n, out);
  return cudaGetLastError();
}

template <int OPT>
__global__ void opt_kernel(OptConsts oc, const float* p, const float* g, const float* s1, const float* s2,
                           int64_t n, float* op, float* os1, float* os2) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float pp = p[i];
    if (OPT == OPT_SGD) {
      float vel = s1 ? s1[i] : 0.0f;
      sgd_elem(pp, g[i], vel, oc);
      if (os1) os1[i] = vel;
    } else if (OPT == OPT_LION || OPT == OPT_ADAGRAD) {
      float st = s1[i];
      if (OPT == OPT_LION)
        lion_elem(pp, g[i], st, oc);
      else
        adagrad_elem(pp, g[i], st, oc);
      os1[i] = st;
    } else if (OPT == OPT_RMSPROP) {
      float sq = s1[i], buf = s2 ? s2[i] : 0.0f;
      rmsprop_elem(pp, g[i], sq, buf, oc);
      os1[i] = sq;
      if (os2) os2[i] = buf;
    } else {
      float m = s1[i], v = s2[i];
      adam_elem<OPT == OPT_ADAMW>(pp, g[i], m, v, oc);
      os1[i] = m;
      os2[i] = v;
    }
    op[i] = pp;
  }
}

cudaError_t launch_opt_step(int opt, const OptConsts& oc, const float* p, const float* g, const float* s1,
                            const float* s2, int64_t n, float* op, float* os1, float* os2, cudaStream_t st) {
  if (opt == OPT_SGD)
    opt_kernel<OPT_SGD><<<grid_for(n), kThreads, 0, st>>>(oc, p, g, s1, s2, n, op, os1, os2);
  else if (opt == OPT_ADAM)
    opt_kernel<OPT_ADAM><<<grid_for(n), kThreads, 0, st>>>(oc, p, g, s1, s2, n, op, os1, os2);
  else if (opt == OPT_ADAMW)
    opt_kernel<OPT_ADAMW><<<grid_for(n), kThreads, 0, st>>>(oc, p, g, s1, s2, n, op, os1, os2);
  else if (opt == OPT_LION)
    opt_kernel<OPT_LION><<<grid_for(n), kThreads, 0, st>>>(oc, p, g, s1, s2, n, op, os1, os2);
  else if (opt == OPT_RMSPROP)
    opt_kernel<OPT_RMSPROP><<<grid_for(n), kThreads, 0, st>>>(oc, p, g, s1, s2, n, op, os1, os2);
  else
    opt_kernel<OPT_ADAGRAD><<<grid_for(n), kThreads, 0, st>>>(oc, p, g, s1, s2, n, op, os1, os2);
  return cudaGetLastError();
}

}  // namespace ody

namespace ody {
// Test hook: div_by against the IEEE division for arbitrary (x, s) pairs.
__global__ void selftest_divide_kernel(const float* x, const float* s, int64_t n, float* fast, float* ieee) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    fast[i] = div_by(x[i], s[i], __frcp_rn(s[i]));
    ieee[i] = __fdiv_rn(x[i], s[i]);
  }
}

cudaError_t launch_selftest_divide(const float* x, const float* s, int64_t n, float* fast, float* ieee,
                                   cudaStream_t st) {
  selftest_divide_kernel<<<grid_for(n), kThreads, 0, st>>>(x, s, n, fast, ieee);
  return cudaGetLastError();
}
}  // namespace ody
