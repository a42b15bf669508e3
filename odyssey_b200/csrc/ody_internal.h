// ody_internal.h -- structures shared between the kernels and the host side
// of libodyssey_mp.so.  Not part of the public C ABI (include/odyssey_mp.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "ody_numerics.cuh"

namespace ody {

// Element tile of the multi-tensor kernels: 256 threads x 8 elements.  Every
// tensor starts on a TILE boundary of its own quantised-output region, so a
// tile's MXFP4 (64 blocks x 17 B = 1088 B) or NVFP4 (128 blocks x 9 B =
// 1152 B) output is one contiguous, 16-byte aligned byte range.
constexpr int kThreads = 256;
constexpr int kVec = 8;
constexpr int kTile = kThreads * kVec;  // 2048 elements
constexpr int kChunk = 32 * kTile;      // 65536 elements per chunk-table entry (at most)
constexpr int kPad = 64;                // arena alignment of every tensor (elements)
constexpr uint32_t kRequantJob = 0x80000000u;  // job-list entry flag: a requant job
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // default bound on a device-side wait (2 s)
constexpr int kMxTileBytes = (kTile / 32) * 17;  // 1088
constexpr int kNvTileBytes = (kTile / 16) * 9;   // 1152

// One parameter tensor inside the flat arenas.
struct TensorDesc {
  int64_t off;     // element offset in the master/state/grad arenas (multiple of kPad)
  int64_t numel;   // real elements
  int64_t npad;    // numel rounded up to kPad
  int64_t qoff;    // byte offset in the quantised-output arena (multiple of 256)
  int32_t quant;   // ody::Q_*
  int32_t nchunks; // update chunks of this tensor
};

// One entry of the chunk table: a kTile-aligned slice of one tensor.
struct Chunk {
  int64_t start;   // element offset in the arenas
  int32_t len;     // elements (a multiple of kTile, or the tensor's padded tail; <= kChunk)
  int32_t tensor;  // index into the TensorDesc table
};

// Loss-scaler state machine kept in device memory so a step needs no host
// round trip (GradientScaler, src/odyssey/training/mixed_precision.mojo:45-237
// and PrecisionConfig counters, precision_config.mojo:455-473).
struct DevScaler {
  float scale;
  float pad;
  int64_t steps_since_growth;
  int64_t num_steps;
  int64_t step_count;
  int64_t overflow_count;
};

struct DecideParams {
  int32_t use_scaler;
  int32_t clip_enabled;
  float max_norm;
  float growth_factor;
  float backoff_factor;
  float min_scale;
  float max_scale;
  int32_t pad;
  int64_t growth_interval;
};

// What pass 1 decided for this step; read by passes 2 and 3 and copied to
// the host as the step result.
struct Decision {
  int32_t skip;
  int32_t clipped;
  float coef;
  float norm;
  float scale_used;
  float scale_next;
  float unscale_div;  // the divisor, the scale rounded to the gradient dtype
  int32_t err;        // set by the apply kernel when a bounded wait ran out
  double sumsq;
  int64_t nonfinite;
  int64_t step_count;
  int64_t overflow_count;
  int64_t scaler_num_steps;
  int64_t steps_since_growth;
};

struct StatsPartial {
  double sumsq;
  int64_t nonfinite;
};

// ---- launchers (ody_kernels.cu) -----------------------------------------
void upload_fp4_tables(int device);  // once per device
cudaError_t launch_stats(int gdt, const void* grad, int64_t n, int use_scaler, DevScaler* scaler,
                         StatsPartial* partials, int grid, unsigned* ticket, int world_mode,
                         double* local_stats, const DecideParams& dp, Decision* dec,
                         uint32_t* amax_slots, uint32_t* sync, int ntensors, cudaStream_t st);
cudaError_t launch_finalize(const double* gathered, int world, DevScaler* scaler,
                            const DecideParams& dp, Decision* dec, uint32_t* amax_slots,
                            int ntensors, cudaStream_t st);
cudaError_t launch_apply(int gdt, int opt, const OptConsts& oc, int use_scaler, const Chunk* chunks,
                         const uint32_t* jobs, int njobs, const TensorDesc* tensors, float* master, float* s1,
                         float* s2, const void* grad, uint8_t* qout, uint32_t* amax_slots, float* qscale,
                         uint32_t* sync, Decision* dec, int grid, cudaStream_t st, unsigned long long wait_ns);
// pass 1 with the data-parallel gradient reduce-scatter fused in (up to 8
// ranks; peers: device array of the ranks' full gradient buffers)
cudaError_t launch_rs_stats(int gdt, const void* const* peers, int world, int64_t shard_off, void* grad, int64_t n,
                            int use_scaler, DevScaler* scaler, StatsPartial* partials, int grid, unsigned* ticket,
                            int world_mode, double* local_stats, const DecideParams& dp, Decision* dec,
                            uint32_t* amax_slots, uint32_t* sync, int ntensors, cudaStream_t st);
cudaError_t launch_fp4_single_encode(int mx, const float* x, int64_t n, const uint64_t* seeds, uint8_t* vals,
                                     uint8_t* scs, cudaStream_t st);
cudaError_t launch_fp4_single_decode(int mx, const uint8_t* vals, const uint8_t* scs, int64_t n, float* out,
                                     cudaStream_t st);
int apply_grid(int gdt, int opt, int device);
// the apply kernel instance for (gdt, opt), and an update of its node in an
// instantiated graph with new launch arguments
const void* apply_kernel_fn(int gdt, int opt);
cudaError_t set_apply_node(cudaGraphExec_t exec, cudaGraphNode_t node, int gdt, int opt, const OptConsts& oc,
                           int use_scaler, const Chunk* chunks, const uint32_t* jobs, int njobs,
                           const TensorDesc* tensors, float* master, float* s1, float* s2, const void* grad,
                           uint8_t* qout, uint32_t* amax_slots, float* qscale, uint32_t* sync, Decision* dec,
                           int grid, unsigned long long wait_ns);
int stats_grid(int device);

// stateless whole-tensor operations (device pointers)
cudaError_t launch_amax(int src_dtype, const void* x, int64_t n, uint32_t* amax, cudaStream_t st);
cudaError_t launch_quantize(int kind, int src_dtype, const void* x, int64_t n, uint8_t* out,
                            const uint32_t* amax, float* tensor_scale, cudaStream_t st);
cudaError_t launch_dequantize(int kind, const uint8_t* q, int64_t n, const float* tensor_scale,
                              float* out, cudaStream_t st);
cudaError_t launch_unscale(int dtype, const void* g, int64_t n, float scale, void* out,
                           cudaStream_t st);
cudaError_t launch_count_nonfinite(int dtype, const void* g, int64_t n,
                                   unsigned long long* count, cudaStream_t st);
cudaError_t launch_sumsq(const float* g, int64_t n, StatsPartial* partials, int grid,
                         unsigned* ticket, double* total, cudaStream_t st);
cudaError_t launch_scale_inplace(float* g, int64_t n, const float* coef, cudaStream_t st);
cudaError_t launch_sumsq64(const float* g, int64_t n, StatsPartial* partials, int grid, unsigned* ticket,
                           double* total, cudaStream_t st);
cudaError_t launch_clip_variant_coef(const double* total, double max_norm, double* norm_out, double* coef,
                                     cudaStream_t st);
cudaError_t launch_clip_variant_scale(float* g, int64_t n, const double* coef, int mode, cudaStream_t st);
cudaError_t launch_clip_coef(const double* total, float max_norm, float* norm_out,
                             float* coef_out, cudaStream_t st);
cudaError_t launch_opt_step(int opt, const OptConsts& oc, const float* p, const float* g,
                            const float* s1, const float* s2, int64_t n, float* op, float* os1,
                            float* os2, cudaStream_t st);

}  // namespace ody

namespace ody {
cudaError_t launch_selftest_divide(const float* x, const float* s, int64_t n, float* fast, float* ieee,
                                   cudaStream_t st);
}

namespace ody {
// sets the message ody_last_error(NULL) returns on this thread
void record_error(const std::string& msg);
}
