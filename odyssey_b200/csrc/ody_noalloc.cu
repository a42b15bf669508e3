// ody_noalloc.cu -- ody_global_norm_clip_noalloc: the global-norm clip
// (clip_gradients_by_global_norm, gradient_clipping.mojo:313-368) for callers
// that must not allocate GPU memory.
//
// Some callers cannot call cudaMalloc or any allocating routine: code that
// runs inside another framework's memory pool with a fixed budget, code
// between the captures of a CUDA graph whose memory is already laid out, or
// real-time callers for which an allocation (and its implicit
// synchronisation) is not allowed.  ody_global_norm_clip stages its
// per-CTA partial sums and its pointer table in buffers it allocates per
// call; this variant keeps all of that in one file-scope __device__ array
// instead, so a call allocates nothing.  The caller still passes the
// gradients (device memory, clipped in place) and receives the norm.
//
// The array (struct NoAllocScratch, about 32 KB) is part of the module, so
// every GPU that loads this library holds it until the process exits.  All
// calls on a device share it and it keeps the last call's contents: a call
// clears what must start at zero itself, and calls that overlap on the GPU
// (from different host threads or streams) race on it.
#include <mutex>
#include <string>

#include "../../include/odyssey_mp.h"
#include "ody_internal.h"

namespace {

constexpr int kNaMaxTensors = 1024;  // per call
constexpr int kNaBlocks = 592;       // CTAs of the reduction (one partial each)
constexpr int kNaThreads = 256;

struct NoAllocScratch {
  const float* ptr[kNaMaxTensors];
  int64_t numel[kNaMaxTensors];
  double partial[kNaBlocks];
  double total;
  unsigned ticket;
  float norm;
  float coef;
  int32_t ntensors;
};

static __device__ __align__(256) NoAllocScratch g_na_scratch;

// float32 squares of 8 consecutive elements reduced in float32 as a width-8
// SIMD reduce_add (halves added pairwise), then accumulated in float64: the
// summation of _norm_sq_simd_f32 (gradient_clipping.mojo:52-67) with 8 lanes,
// the same grouping as ody_global_norm_clip.
__device__ __forceinline__ float na_sq8(const float* g, int64_t i, int64_t n) {
  float q[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float x = (i + k < n) ? g[i + k] : 0.0f;
    q[k] = __fmul_rn(x, x);
  }
  const float a0 = __fadd_rn(q[0], q[4]), a1 = __fadd_rn(q[1], q[5]);
  const float a2 = __fadd_rn(q[2], q[6]), a3 = __fadd_rn(q[3], q[7]);
  return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}

__device__ __forceinline__ double na_block_sum(double v) {
  __shared__ double sm[kNaThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < kNaThreads / 32 ? sm[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  __syncthreads();
  return v;
}

// Pass 1: per-CTA partial sums over all tensors of the table; the last CTA
// adds the partials in CTA order (deterministic) and forms the norm and the
// clip coefficient (gradient_clipping.mojo:310,352).
__global__ void __launch_bounds__(kNaThreads) na_sumsq_kernel(float max_norm) {
  NoAllocScratch& S = g_na_scratch;
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int t = 0; t < S.ntensors; t++) {
    const float* g = S.ptr[t];
    const int64_t n = S.numel[t];
    const int64_t ng = (n + 7) / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < ng; i += stride)
      acc += (double)na_sq8(g, i * 8, n);
  }
  acc = na_block_sum(acc);
  __shared__ bool last;
  if (threadIdx.x == 0) {
    S.partial[blockIdx.x] = acc;
    __threadfence();
    last = atomicAdd(&S.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  double s = 0.0;
  for (int j = threadIdx.x; j < (int)gridDim.x; j += blockDim.x) s += __ldcg(&S.partial[j]);
  s = na_block_sum(s);
  if (threadIdx.x == 0) {
    S.total = s;
    const float norm = __double2float_rn(__dsqrt_rn(s));
    S.norm = norm;
    S.coef = norm > max_norm ? __double2float_rn(__ddiv_rn((double)max_norm, __dadd_rn((double)norm, 1e-6)))
                             : 1.0f;
  }
}

// Pass 2: g = g * Float32(coef) in place when the norm exceeded max_norm
// (_scale_simd_f32, gradient_clipping.mojo:88-101).
__global__ void __launch_bounds__(kNaThreads) na_scale_kernel() {
  NoAllocScratch& S = g_na_scratch;
  const float c = S.coef;
  if (c == 1.0f) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int t = 0; t < S.ntensors; t++) {
    float* g = const_cast<float*>(S.ptr[t]);
    const int64_t n = S.numel[t];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
      g[i] = __fmul_rn(g[i], c);
  }
}

// Device address of g_na_scratch, looked up once per device with that device
// current (in host code the symbol is only a host-side stand-in).
std::mutex g_na_mu;
void* g_na_addr[64] = {nullptr};

int na_fail(int code, const std::string& msg) {
  ody::record_error(msg);  // reported by ody_last_error(NULL)
  return code;
}

}  // namespace

extern "C" int ody_global_norm_clip_noalloc(float* const* grads, const int64_t* numels, int32_t ntensors,
                                            float max_norm, float* total_norm) {
  if (!(max_norm > 0.0f))
    return na_fail(ODY_ERR_ARG, "max_norm must be positive, got: " + std::to_string(max_norm));
  if (ntensors < 0 || (ntensors > 0 && (!grads || !numels)))
    return na_fail(ODY_ERR_ARG, "ody_global_norm_clip_noalloc: bad tensor list");
  if (ntensors > kNaMaxTensors)
    return na_fail(ODY_ERR_SHAPE, "ody_global_norm_clip_noalloc: at most " + std::to_string(kNaMaxTensors) +
                                      " tensors per call, got " + std::to_string(ntensors));
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail(ODY_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return na_fail(ODY_ERR_ARG, "device ordinal out of range");
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_addr[dev]) {
      e = cudaGetSymbolAddress(&g_na_addr[dev], g_na_scratch);
      if (e != cudaSuccess) {
        g_na_addr[dev] = nullptr;
        return na_fail(ODY_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      }
    }
    base = g_na_addr[dev];
  }
  NoAllocScratch* S = static_cast<NoAllocScratch*>(base);
  // the table goes into the scratch array from host stack memory: no allocation
  const float* ptrs[kNaMaxTensors];
  int64_t ns[kNaMaxTensors];
  for (int i = 0; i < ntensors; i++) {
    if (numels[i] < 0 || (numels[i] > 0 && !grads[i]))
      return na_fail(ODY_ERR_ARG, "ody_global_norm_clip_noalloc: bad tensor " + std::to_string(i));
    cudaPointerAttributes a;
    if (numels[i] > 0) {
      if (cudaPointerGetAttributes(&a, grads[i]) != cudaSuccess ||
          (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)) {
        cudaGetLastError();
        return na_fail(ODY_ERR_ARG, "ody_global_norm_clip_noalloc: gradient " + std::to_string(i) +
                                        " is not device memory");
      }
      // another GPU's memory: without peer access the kernels below would
      // fault on it, so it is refused before anything is launched
      if (a.type == cudaMemoryTypeDevice && a.device != dev)
        return na_fail(ODY_ERR_ARG, "ody_global_norm_clip_noalloc: gradient " + std::to_string(i) +
                                        " is memory of GPU " + std::to_string(a.device) +
                                        ", not of the current GPU " + std::to_string(dev));
    }
    ptrs[i] = grads[i];
    ns[i] = numels[i];
  }
  const cudaStream_t st = cudaStreamPerThread;
  const int32_t nt = ntensors;
#define NA_CUDA(call)                                                                  \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess) return na_fail(ODY_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)
  if (nt > 0) {
    NA_CUDA(cudaMemcpyAsync(S->ptr, ptrs, sizeof(float*) * nt, cudaMemcpyHostToDevice, st));
    NA_CUDA(cudaMemcpyAsync(S->numel, ns, sizeof(int64_t) * nt, cudaMemcpyHostToDevice, st));
  }
  NA_CUDA(cudaMemcpyAsync(&S->ntensors, &nt, sizeof(nt), cudaMemcpyHostToDevice, st));
  NA_CUDA(cudaMemsetAsync(&S->ticket, 0, sizeof(unsigned), st));
  na_sumsq_kernel<<<kNaBlocks, kNaThreads, 0, st>>>(max_norm);
  NA_CUDA(cudaGetLastError());
  na_scale_kernel<<<kNaBlocks, kNaThreads, 0, st>>>();
  NA_CUDA(cudaGetLastError());
  float hn = 0.0f;
  NA_CUDA(cudaMemcpyAsync(&hn, &S->norm, sizeof(float), cudaMemcpyDeviceToHost, st));
  NA_CUDA(cudaStreamSynchronize(st));
#undef NA_CUDA
  if (total_norm) *total_norm = hn;
  return ODY_OK;
}
