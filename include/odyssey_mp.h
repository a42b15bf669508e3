/*
 * odyssey_mp.h -- C ABI of libodyssey_mp.so, the B200 (sm_100a) mixed-
 * precision parameter-update path of Odyssey.
 *
 * Plain C types only (pointers, sizes, POD structs); no CUDA or PyTorch
 * types appear in a signature.  Every entry point returns an int status
 * (ODY_OK or a negative ODY_ERR_*); the message of the last failure is
 * returned by ody_last_error().  Where the reference raises an Error the
 * message text is the reference's.
 *
 * Each declaration names the reference interface (HomericIntelligence/
 * Odyssey, Mojo; file:line inside that project) it replaces.  A pointer
 * argument of the stateless single-op functions may be host or device
 * memory (detected per call); context buffers live in device memory owned by
 * the context.
 */
#ifndef ODYSSEY_MP_H
#define ODYSSEY_MP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ODY_ABI_VERSION 1

/* ---- status codes -------------------------------------------------------- */
#define ODY_OK 0
#define ODY_ERR_ARG (-1)
#define ODY_ERR_SHAPE (-2)
#define ODY_ERR_DTYPE (-3)
#define ODY_ERR_CUDA (-4)
#define ODY_ERR_NCCL (-5)
#define ODY_ERR_COMM_TIMEOUT (-6)
#define ODY_ERR_DEVICE_BOUNDS (-7)
#define ODY_ERR_STATE (-8)

/* ---- element dtypes of gradients (DType.float32/float16/bfloat16) -------- */
#define ODY_F32 0
#define ODY_F16 1
#define ODY_BF16 2

/* ---- optimizers (src/odyssey/training/optimizers/<name>.mojo) ------------- */
#define ODY_SGD 0      /* sgd.mojo */
#define ODY_ADAM 1     /* adam.mojo */
#define ODY_ADAMW 2    /* adamw.mojo */
#define ODY_LION 3     /* lion.mojo: state m; beta1/beta2 as Lion's (0.9 / 0.99 there) */
#define ODY_RMSPROP 4  /* rmsprop.mojo: state square_avg (+ buf with momentum > 0); alpha */
#define ODY_ADAGRAD 5  /* adagrad.mojo: state accum; its default epsilon is 1e-10 */

/* ---- re-quantisation targets of the updated master weights --------------- */
#define ODY_Q_NONE 0
#define ODY_Q_FP16 1           /* update_model_from_master, FP16 (mixed_precision.mojo:299-354) */
#define ODY_Q_BF16 2           /* update_model_from_master, BF16 */
#define ODY_Q_FP8_E4M3 3       /* AnyTensor.to_fp8() (any_tensor.mojo:1946) */
#define ODY_Q_FP8_E5M2 4       /* AnyTensor.to_bf8() (any_tensor.mojo:2165) */
#define ODY_Q_FP8_E4M3_TENSOR 5 /* e4m3(w / s), s = amax/448 (per-tensor scale; extension) */
#define ODY_Q_MXFP4 6          /* AnyTensor.to_mxfp4() (any_tensor.mojo:2237-2302), 17-byte blocks */
#define ODY_Q_NVFP4 7          /* AnyTensor.to_nvfp4() (any_tensor.mojo:2329-2401), 9-byte blocks */
#define ODY_Q_NVFP4_TENSOR 8   /* to_nvfp4(w / s_t), s_t = amax/(448*6) (per-tensor scale; extension) */
/* MXFP4 by the OCP Microscaling Formats v1.0 rule (no reference counterpart;
 * the rule BASELINE's MXFP4 configuration states): per 32-element block the
 * E8M0 byte X + 127 with X = floor(log2(max|x|)) - 2 clamped to [-127, 127],
 * elements x / 2^X rounded to nearest even on the E2M1 grid (0.5 included)
 * and saturated at 6, sign kept; a NaN or Inf element gives the NaN scale
 * byte 0xFF.  Same 17-byte block layout as ODY_Q_MXFP4.  Stateless
 * quantise / dequantise only (not a step context requant kind). */
#define ODY_Q_MXFP4_OCP 9

/* ---- requant job placement (ody_config.requant_placement) ---------------
 * INTERLEAVED: a tensor's requant jobs follow its last update job by two
 * grid-widths of jobs, two per update job of the tensors after it; a
 * tensor with fewer than two grid-widths of update jobs after it has its
 * requant jobs at the end.  AT_END: all requant jobs after all update jobs.
 * AUTO: INTERLEAVED.  Results are identical under every placement. */
#define ODY_REQUANT_AUTO 0
#define ODY_REQUANT_INTERLEAVED 1
#define ODY_REQUANT_AT_END 2

/* ---- context buffers ------------------------------------------------------ */
#define ODY_BUF_MASTER 0 /* float32 master weights */
#define ODY_BUF_STATE1 1 /* SGD velocity / Adam(W) first moment m (float32) */
#define ODY_BUF_STATE2 2 /* Adam(W) second moment v (float32) */
#define ODY_BUF_GRAD 3   /* scaled gradients, in the context's gradient dtype */
/* with data-parallel gradients attached: tensor index's slice of this rank's
 * full-model gradient buffer (any tensor, owned or not) */
#define ODY_BUF_DP_GRAD 4

/*
 * Step configuration.  Field names follow the reference: optimizer hyper-
 * parameters are Float64 exactly as sgd_step/adam_step/adamw_step take them
 * (sgd.mojo:27-35, adam.mojo:42-53, adamw.mojo:44-55); the scaler fields
 * are GradientScaler.__init__'s (mixed_precision.mojo:96-122) and the TOML
 * keys [precision.gradient_scaler] / [precision.gradient_clipping]
 * (configs/lenet5/emnist/fp16.toml).
 */
typedef struct ody_config {
  int32_t optimizer;          /* ODY_SGD ... ODY_ADAGRAD */
  int32_t device;             /* CUDA device ordinal */
  double learning_rate;
  double momentum;            /* SGD, RMSprop */
  double beta1, beta2, epsilon; /* Adam / AdamW / Lion (betas), RMSprop / Adagrad (epsilon) */
  double weight_decay;
  int32_t use_gradient_scaler;  /* PrecisionConfig.use_gradient_scaler */
  float initial_scale;          /* default 65536 */
  float growth_factor;          /* default 2.0 */
  float backoff_factor;         /* default 0.5 */
  int64_t growth_interval;      /* default 2000 */
  float min_scale;              /* default 1.0 */
  float max_scale;              /* default 65536 */
  int32_t clip_enabled;         /* clip_gradients_by_global_norm */
  float max_norm;
  int32_t comm_timeout_ms;      /* multi-GPU: bound on every collective wait */
  int32_t reserved0;
  double alpha;                 /* RMSprop smoothing constant (default 0.99) */
  int32_t chunk_elems;          /* apply-job chunk length in elements, a multiple of 2048 up to
                                   65536; 0 (default): chosen from the model size */
  int32_t requant_placement;    /* where the per-tensor-scaled kinds' requant jobs run inside the
                                   apply kernel: ODY_REQUANT_AUTO (default), _INTERLEAVED, _AT_END */
  int32_t reserved[2];
} ody_config;

/* What one step did (PrecisionConfig.step bookkeeping,
 * precision_config.mojo:455-473, plus the clip of gradient_clipping.mojo:313-368). */
typedef struct ody_step_result {
  int32_t found_inf;      /* any non-finite unscaled gradient (all ranks) */
  int32_t skipped;        /* update skipped (== found_inf) */
  int32_t clipped;        /* global norm exceeded max_norm */
  int32_t reserved0;
  int64_t nonfinite_count;
  double sumsq;           /* sum of float32 squares of the unscaled gradients */
  float grad_norm;        /* Float32(sqrt(sumsq)) (gradient_clipping.mojo:310) */
  float clip_coef;        /* 1.0 when not clipped */
  float scale_used;       /* loss scale this step's gradients were unscaled by */
  float scale_next;       /* loss scale after step()/backoff() */
  int64_t step_count;     /* PrecisionConfig._step_count */
  int64_t overflow_count; /* PrecisionConfig._overflow_count */
  int64_t scaler_num_steps;   /* GradientScaler._num_steps */
  int64_t steps_since_growth; /* GradientScaler._steps_since_growth */
} ody_step_result;

typedef struct ody_ctx ody_ctx;

/* ---- library ------------------------------------------------------------- */
int ody_abi_version(void);
/* Message of the last failure on this thread (ctx may be NULL). */
const char* ody_last_error(const ody_ctx* ctx);
/* Fills the reference defaults: GradientScaler() (mixed_precision.mojo:
 * 96-122), AdamW betas/eps (adamw.mojo:44-55), clip disabled. */
void ody_config_default(ody_config* cfg);
/* Bytes of the quantised form of n elements (tensor_dtype_conv.mojo:281-366). */
int64_t ody_quant_bytes(int32_t kind, int64_t n);

/* ---- the fused step context (replaces PrecisionConfig + GradientScaler +
 *      init_*_state + the per-tensor optimizer/requant call sequence of
 *      examples/lenet_emnist/run_train.mojo:219-306 and
 *      examples/mixed_precision_training.mojo:132-216) ----------------------- */
int ody_ctx_create(ody_ctx** out, const ody_config* cfg);
/* Registers one parameter tensor (in model order); *index_out receives its
 * global index.  All tensors of a context share one gradient dtype.
 * Replaces init_optimizer_state (dispatch.mojo:227-313): states start at 0. */
int ody_ctx_add_tensor(ody_ctx* ctx, int64_t numel, int32_t grad_dtype, int32_t quant_kind,
                       int32_t* index_out);
/* Freezes the tensor list, assigns whole tensors to ranks (ZeRO-1 flat
 * shard; see ody_plan_shards), allocates this rank's device arenas and, for
 * world_size > 1, joins the NCCL communicator identified by the 128-byte
 * nccl_unique_id (from ody_nccl_unique_id on rank 0). */
int ody_ctx_finalize(ody_ctx* ctx, int32_t world_size, int32_t rank, const void* nccl_unique_id);
/* 128-byte NCCL unique id for ody_ctx_finalize (call on one rank, share it). */
int ody_nccl_unique_id(void* out128);
/* Host-only: contiguous balanced assignment of whole tensors to ranks (by
 * element count).  owner_out[i] = rank owning tensor i. */
int ody_plan_shards(const int64_t* numels, int32_t ntensors, int32_t world_size, int32_t* owner_out);
int ody_ctx_tensor_owner(const ody_ctx* ctx, int32_t index, int32_t* rank_out);
int ody_ctx_num_tensors(const ody_ctx* ctx, int32_t* n_out);

/* Copy one tensor's buffer in / out (host or device memory; bytes must be
 * numel * element size).  Synchronous. */
int ody_upload(ody_ctx* ctx, int32_t which, int32_t index, const void* src, size_t bytes);
int ody_download(ody_ctx* ctx, int32_t which, int32_t index, void* dst, size_t bytes);
/* As ody_upload, enqueued on the context stream without waiting; the source
 * must stay valid (and, for overlap, be pinned) until the next synchronous
 * call on the context. */
int ody_upload_async(ody_ctx* ctx, int32_t which, int32_t index, const void* src, size_t bytes);
/* Device address of one tensor inside a context arena (zero-copy producers). */
int ody_ctx_device_ptr(ody_ctx* ctx, int32_t which, int32_t index, void** ptr_out);
/* The context's CUDA stream as an opaque handle. */
int ody_ctx_stream(ody_ctx* ctx, void** stream_out);

/* One fused step: unscale -> finite check -> [skip + backoff] -> clip ->
 * optimizer -> requant -> scaler step.  t is the optimizer timestep
 * (>= 1 for Adam/AdamW, adam.mojo:117-118).  Synchronous; fills *out. */
int ody_step(ody_ctx* ctx, int64_t t, ody_step_result* out);
/* Enqueue a step without waiting; ody_step_wait returns its result. */
int ody_step_async(ody_ctx* ctx, int64_t t);
int ody_step_wait(ody_ctx* ctx, ody_step_result* out);

/* Per-pass device timing (no reference counterpart; used for the roofline):
 * when enabled, every step records CUDA events on the context stream around
 * pass 1 (gradient statistics), the multi-GPU exchange, pass 2 (update) and
 * pass 3 (per-tensor requant).  ody_ctx_pass_times waits for the stream and
 * returns the accumulated milliseconds per pass (ms_out[4]) and the number
 * of timed steps, then resets the accumulators. */
int ody_ctx_set_timing(ody_ctx* ctx, int32_t enable);
int ody_ctx_pass_times(ody_ctx* ctx, double* ms_out, int64_t* steps_out);

/* Graph mode (one GPU): the first step after enabling captures the step's
 * launches (stats, apply, result read-back) into one CUDA graph; later steps
 * replay it with one graph launch, updating only the optimizer constants of
 * step t.  Host launch overhead per step drops to one graph launch, which is
 * what bounds small models (LeNet: 61,706 params).  Ignored while per-pass
 * timing is on, while gradients are double-buffered, and with world_size > 1
 * (the NCCL exchange stays eager).
 * The reference has no equivalent (its step is a CPU call); results are
 * identical to the eager path. */
int ody_ctx_set_graph(ody_ctx* ctx, int32_t enable);

/* Double-buffered gradients (no reference counterpart; the reference's step
 * reads host tensors).  Enabling allocates a second gradient arena.  From
 * then on ODY_BUF_GRAD names the arena the NEXT step reads; ody_upload /
 * ody_upload_async into it run on a separate copy stream, ordered after the
 * step that last read that arena, and the step waits for them.  The arenas
 * alternate with every step, so the host can queue step t+1's gradient
 * upload right after ody_step_async(t) and the copy overlaps step t's
 * kernels: a host-fed loop then runs at the rate of the slower of the PCIe
 * copy and the kernels rather than their sum.  ody_ctx_device_ptr(...,
 * ODY_BUF_GRAD, ...) also names the next step's arena, which changes with
 * every step.  Graph mode is not used while this is on (steps run eagerly),
 * and it does not combine with ody_ctx_dp_attach.  Disabling keeps the arena
 * the next step would have read. */
int ody_ctx_set_grad_double_buffer(ody_ctx* ctx, int32_t enable);

/* Data-parallel gradients (collective over the context's ranks, at most 8).
 * Allocates this rank's full-model gradient buffer (every tensor, in the
 * context's gradient dtype, padded like the arenas; filled through
 * ODY_BUF_DP_GRAD) and maps every other rank's buffer here through CUDA IPC
 * (peer access over NVLink).  From then on each step starts with the
 * gradient reduce-scatter fused into pass 1: this rank's shard is summed
 * over all ranks in float32 in rank order, rounded once to the gradient
 * dtype, written to the shard's gradient arena and its statistics taken in
 * the same kernel.  The sum (not the mean) is the gradient; fold 1/N into
 * the loss scale for a mean.  The reference is single-process, so this
 * extends its step to data-parallel training
 * (examples/mixed_precision_training.mojo:132-216 with per-rank backward). */
int ody_ctx_dp_attach(ody_ctx* ctx);

/* Quantised weights of one tensor in the reference's byte layout, and its
 * per-tensor scale (1.0 for kinds without one). */
int ody_get_quant(ody_ctx* ctx, int32_t index, void* dst, size_t bytes, float* tensor_scale);
/* The full low-precision model after a sharded step (ZeRO-1's consumer; the
 * reference holds the whole model in one process, so the layout is that of
 * AnyTensor.to_* per tensor, tensor_dtype_conv.mojo:281-366).  The gathered
 * buffer holds every tensor's quantised region in global order;
 * ody_ctx_quant_layout gives tensor index's byte offset in it and its
 * meaningful bytes (ody_quant_bytes), and *total the buffer size
 * (index < 0: total only). */
int ody_ctx_quant_layout(const ody_ctx* ctx, int32_t index, int64_t* offset, int64_t* bytes, int64_t* total);
/* Every rank's quantised weights and per-tensor scales into every rank's
 * dst (device, *total bytes) and scales (device, one float per tensor):
 * one NCCL broadcast per rank of its contiguous slice, grouped.  Collective:
 * all ranks call it.  Synchronous, bounded by comm_timeout_ms. */
int ody_ctx_gather_quant(ody_ctx* ctx, void* dst, float* scales);
/* GradientScaler state (mixed_precision.mojo:77-93). */
int ody_get_scaler(ody_ctx* ctx, float* scale, int64_t* steps_since_growth, int64_t* num_steps,
                   int64_t* step_count, int64_t* overflow_count);
int ody_set_scaler(ody_ctx* ctx, float scale, int64_t steps_since_growth, int64_t num_steps,
                   int64_t step_count, int64_t overflow_count);
/* Checkpoint of this rank's master weights, states and scaler
 * (training/checkpoint.mojo:70 CheckpointManager; the reference does not
 * persist the scaler, test_precision_checkpoint.mojo:202-232).  buf NULL ->
 * *bytes receives the size needed. */
int ody_ctx_export(ody_ctx* ctx, void* buf, size_t* bytes);
int ody_ctx_import(ody_ctx* ctx, const void* buf, size_t bytes);
void ody_ctx_destroy(ody_ctx* ctx);

/* ---- stateless single operations (host or device pointers) -------------- */
/* GradientScaler.unscale_gradients (mixed_precision.mojo:154-182). */
int ody_unscale(const void* grads, int32_t dtype, int64_t n, float scale, void* out);
/* check_gradients_finite (mixed_precision.mojo:357-381); *finite = 1 if no NaN/Inf. */
int ody_check_finite(const void* grads, int32_t dtype, int64_t n, int32_t* finite);
/* convert_to_fp32_master (mixed_precision.mojo:240-296). */
int ody_to_fp32(const void* x, int32_t dtype, int64_t n, float* out);
/* clip_gradients_by_global_norm (gradient_clipping.mojo:313-368): float32
 * gradients clipped in place; returns the pre-clip norm in *total_norm. */
int ody_global_norm_clip(float* const* grads, const int64_t* numels, int32_t ntensors, float max_norm,
                         float* total_norm);
/* As ody_global_norm_clip, for callers that cannot allocate GPU memory (a
 * fixed memory budget inside another framework's pool, work placed between
 * graph captures, real-time code where an allocation's implicit
 * synchronisation is not allowed).  No counterpart in the reference.
 * Allocates nothing: its pointer table, per-block partial sums and results
 * live in one file-scope __device__ array of about 32 KB, which every GPU
 * that loads this library holds until the process exits.  grads must be
 * device pointers of the calling thread's current GPU (clipped in place;
 * another GPU's memory is refused with ODY_ERR_ARG); at most 1024 tensors
 * per call, more is rejected with ODY_ERR_SHAPE.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture.  All calls on a device
 * share the array, which keeps the last call's contents (each call clears
 * what must start at zero); calls that overlap on the GPU race.  Runs on
 * the calling thread's per-thread default stream and returns after it
 * completes.  That stream is ordered with the legacy default stream but not
 * with the caller's non-blocking streams (a PyTorch side stream, say):
 * finish or synchronise the stream that produced grads before the call. */
int ody_global_norm_clip_noalloc(float* const* grads, const int64_t* numels, int32_t ntensors,
                                 float max_norm, float* total_norm);
/* The two other global-norm clips of the reference, in place on float32
 * tensors, returning the float64 norm before clipping:
 *   mode 0: clip_grad_global_norm_ (core/numerical_safety.mojo:760-815):
 *           float32 squares, no +1e-6, factor max_norm/norm as float32;
 *   mode 1: clip_global_norm (training/optimizers/optimizer_utils.mojo:
 *           303-348): float64 squares, each value scaled in float64 and
 *           rounded to float32.
 * Both clip only when norm > max_norm and norm > 0; max_norm 0 is allowed.
 * The float64 sums run in a different order than the reference's serial
 * loops (same value to ~1e-15 relative). */
int ody_clip_global_norm_variant(float* const* grads, const int64_t* numels, int32_t ntensors,
                                 double max_norm, int32_t mode, double* total_norm);
/* sgd_step (sgd.mojo:27-121); velocity/out_velocity may be NULL when momentum == 0. */
int ody_sgd_step(const float* params, const float* grads, const float* velocity, int64_t n,
                 double learning_rate, double momentum, double weight_decay, float* out_params,
                 float* out_velocity);
/* adam_step (adam.mojo:42-166). */
int ody_adam_step(const float* params, const float* grads, const float* m, const float* v, int64_t n,
                  int64_t t, double learning_rate, double beta1, double beta2, double epsilon,
                  double weight_decay, float* out_params, float* out_m, float* out_v);
/* adamw_step (adamw.mojo:44-175). */
int ody_adamw_step(const float* params, const float* grads, const float* m, const float* v, int64_t n,
                   int64_t t, double learning_rate, double beta1, double beta2, double epsilon,
                   double weight_decay, float* out_params, float* out_m, float* out_v);
/* FP4 singles: each value with its own power-of-two scale (MXFP4 /
 * NVFP4.from_float32, mxfp4.mojo:303-342, nvfp4.mojo:290-328; with seeds,
 * from_float32_stochastic, mxfp4.mojo:344-396 + 398-483).  kind is
 * ODY_Q_MXFP4 (E8M0 scale bytes) or ODY_Q_NVFP4 (E4M3 scale bytes); values
 * receive the 4-bit E2M1 codes, one per byte.  seeds: NULL for round to
 * nearest, else one seed per value. */
int ody_fp4_single_encode(int32_t kind, const float* x, int64_t n, const uint64_t* seeds, uint8_t* values,
                          uint8_t* scales);
/* MXFP4 / NVFP4.to_float32 (mxfp4.mojo:484-491, nvfp4.mojo:474-481). */
int ody_fp4_single_decode(int32_t kind, const uint8_t* values, const uint8_t* scales, int64_t n, float* out);
/* lion_step (lion.mojo:36-104): returns params and momentum. */
int ody_lion_step(const float* params, const float* grads, const float* m, int64_t n, double learning_rate,
                  double beta1, double beta2, double weight_decay, float* out_params, float* out_m);
/* rmsprop_step (rmsprop.mojo:30-175); buf / out_buf only with momentum > 0
 * (buf NULL: a zero buffer, as the reference initialises it). */
int ody_rmsprop_step(const float* params, const float* grads, const float* square_avg, const float* buf,
                     int64_t n, int64_t t, double learning_rate, double alpha, double epsilon,
                     double weight_decay, double momentum, float* out_params, float* out_square_avg,
                     float* out_buf);
/* adagrad_step (adagrad.mojo:30-120). */
int ody_adagrad_step(const float* params, const float* grads, const float* accum, int64_t n,
                     double learning_rate, double epsilon, double weight_decay, float* out_params,
                     float* out_accum);
/* AnyTensor.to_fp8/to_bf8/to_mxfp4/to_nvfp4 (+ per-tensor-scaled kinds,
 * + FP16/BF16 casts): src is float32 (src_dtype ODY_F32) or bfloat16
 * (ODY_BF16, upcast exactly first); out holds ody_quant_bytes(kind, n)
 * bytes; *tensor_scale (may be NULL) receives the per-tensor scale. */
int ody_quantize(int32_t kind, const void* src, int32_t src_dtype, int64_t n, void* out,
                 float* tensor_scale);
/* AnyTensor.from_fp8/from_bf8/from_mxfp4/from_nvfp4 (tensor_dtype_conv.mojo:
 * 69-92,211-235,369-494): n float32 values out. */
int ody_dequantize(int32_t kind, const void* q, int64_t n, float tensor_scale, float* out);

/* The same two operations stream-ordered on device memory only: no staging,
 * no synchronisation (for quantising inside a CUDA pipeline).  For the
 * per-tensor-scaled kinds, tensor_scale (device float, written) and
 * amax_scratch (device, 8 bytes: the tensor's amax and smallest nonzero
 * magnitude, reset by the call) are required; else both
 * may be NULL.  stream NULL is the legacy default stream. */
int ody_quantize_on_stream(int32_t kind, const void* src, int32_t src_dtype, int64_t n, void* out,
                           float* tensor_scale, uint32_t* amax_scratch, void* stream);
int ody_dequantize_on_stream(int32_t kind, const void* q, int64_t n, const float* tensor_scale, float* out,
                             void* stream);
/* Per-format entry points of the two calls above (same arguments without
 * the kind; the per-tensor-scaled kinds keep the generic calls). */
int ody_quant_mxfp4(const void* src, int32_t src_dtype, int64_t n, void* out);   /* AnyTensor.to_mxfp4 (any_tensor.mojo:2237-2302) */
int ody_quant_nvfp4(const void* src, int32_t src_dtype, int64_t n, void* out);   /* AnyTensor.to_nvfp4 (any_tensor.mojo:2329-2401) */
int ody_quant_fp8_e4m3(const void* src, int32_t src_dtype, int64_t n, void* out);   /* AnyTensor.to_fp8 (any_tensor.mojo:1946) */
int ody_quant_fp8_e5m2(const void* src, int32_t src_dtype, int64_t n, void* out);   /* AnyTensor.to_bf8 (any_tensor.mojo:2165) */
int ody_quant_fp16(const void* src, int32_t src_dtype, int64_t n, void* out);   /* update_model_from_master to FP16 (mixed_precision.mojo:299-354) */
int ody_quant_bf16(const void* src, int32_t src_dtype, int64_t n, void* out);   /* update_model_from_master to BF16 */
int ody_dequant_mxfp4(const void* q, int64_t n, float* out);   /* from_mxfp4 (tensor_dtype_conv.mojo:369-430) */
int ody_dequant_nvfp4(const void* q, int64_t n, float* out);   /* from_nvfp4 (tensor_dtype_conv.mojo:433-494) */
int ody_dequant_fp8_e4m3(const void* q, int64_t n, float* out);   /* from_fp8 (tensor_dtype_conv.mojo:69-92) */
int ody_dequant_fp8_e5m2(const void* q, int64_t n, float* out);   /* from_bf8 (tensor_dtype_conv.mojo:211-235) */
int ody_dequant_fp16(const void* q, int64_t n, float* out);   /* the exact FP16 -> float32 upcast */
int ody_dequant_bf16(const void* q, int64_t n, float* out);   /* the exact BF16 -> float32 upcast */

#ifdef __cplusplus
}
#endif
#endif /* ODYSSEY_MP_H */
