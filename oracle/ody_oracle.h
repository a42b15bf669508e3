/*
 * ody_oracle.h -- CPU restatement of Odyssey's mixed-precision update path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the correctness oracle (and the timed
 * CPU baseline of bench.py's reference arm).  It is never linked into, or
 * called by, the product library (libodyssey_mp.so); only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.
 *
 * Every function restates one piece of the reference (HomericIntelligence/
 * Odyssey, Mojo, CPU-only) with the exact operation order and rounding of
 * the reference; the citations are paths inside that project.
 *
 * Pinning: the optimizer formulas are pinned by the reference's own golden
 * vectors (tests/odyssey/training/optimizers/test_{sgd,adam,adamw,lion,
 * rmsprop}.mojo, float64, tol 1e-9; Adagrad has no reference fixture and is
 * pinned by this restatement of adagrad.mojo only); the scaler by tests/odyssey/training/
 * test_mixed_precision.mojo; the FP4 block formats only by the reference's
 * tolerance tests (tests/core/types/test_{mx,nv}fp4_block.mojo) -- the bit
 * patterns of FP4 codes and scales are pinned by this restatement of
 * src/odyssey/core/types/{mxfp4,nvfp4}.mojo, not by a reference fixture.
 * The FP16/BF16/FP8 element casts come from the Mojo 1.0.0b2 stdlib
 * (not vendored); they are restated as IEEE round-to-nearest-even and
 * cross-checked against torch's CPU casts.
 */
#ifndef ODY_ORACLE_H
#define ODY_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element dtypes (same codes as include/odyssey_mp.h) */
enum { ORA_F32 = 0, ORA_F16 = 1, ORA_BF16 = 2 };
/* optimizers */
enum { ORA_SGD = 0, ORA_ADAM = 1, ORA_ADAMW = 2, ORA_LION = 3, ORA_RMSPROP = 4, ORA_ADAGRAD = 5 };
/* re-quantisation targets (same codes as include/odyssey_mp.h) */
enum {
  ORA_Q_NONE = 0,
  ORA_Q_FP16 = 1,
  ORA_Q_BF16 = 2,
  ORA_Q_FP8_E4M3 = 3,        /* AnyTensor.to_fp8(), no scale          */
  ORA_Q_FP8_E5M2 = 4,        /* AnyTensor.to_bf8(), no scale          */
  ORA_Q_FP8_E4M3_TENSOR = 5, /* e4m3(w / s), s = amax/448             */
  ORA_Q_MXFP4 = 6,           /* AnyTensor.to_mxfp4()                  */
  ORA_Q_NVFP4 = 7,           /* AnyTensor.to_nvfp4()                  */
  ORA_Q_NVFP4_TENSOR = 8,    /* to_nvfp4(w / s_t), s_t = amax/2688    */
  ORA_Q_MXFP4_OCP = 9        /* OCP MX rule: X = floor(log2 amax) - 2, RNE */
};

/* ---- scalar casts ------------------------------------------------------ */
uint16_t ora_f32_to_f16(float x);
float ora_f16_to_f32(uint16_t h);
uint16_t ora_f32_to_bf16(float x);
float ora_bf16_to_f32(uint16_t h);
uint8_t ora_f32_to_e4m3(float x); /* RNE, saturating to +-448, NaN -> 0x7F */
float ora_e4m3_to_f32(uint8_t b);
uint8_t ora_f32_to_e5m2(float x); /* RNE, saturating to +-57344, NaN -> 0x7F */
float ora_e5m2_to_f32(uint8_t b);

/* ---- FP4 block pieces (mxfp4.mojo / nvfp4.mojo) ------------------------- */
uint8_t ora_e8m0_from_f32(float scale);
float ora_e8m0_to_f32(uint8_t e);
uint8_t ora_e4m3_scale_from_f32(float scale);
uint8_t ora_fp4_from_f32(float x, float scale);
float ora_fp4_to_f32(uint8_t code, float scale);
void ora_mxfp4_block_encode(const float v[32], uint8_t out[17]);
void ora_mxfp4_block_decode(const uint8_t in[17], float v[32]);
void ora_nvfp4_block_encode(const float v[16], uint8_t out[9]);
void ora_nvfp4_block_decode(const uint8_t in[9], float v[16]);

/* ---- tensor-level quantisation (tensor_dtype_conv.mojo) ----------------- */
int64_t ora_quant_bytes(int kind, int64_t numel);
/* x: n float32 values; out: ora_quant_bytes(kind, n) bytes.  Returns the
 * per-tensor scale (1.0 for kinds without one). */
float ora_quantize(int kind, const float* x, int64_t n, uint8_t* out);
void ora_dequantize(int kind, const uint8_t* q, int64_t n, float tensor_scale,
                    float* out);

/* ---- loss scaler (mixed_precision.mojo:45-237) -------------------------- */
typedef struct {
  float scale, growth_factor, backoff_factor, min_scale, max_scale;
  int64_t growth_interval, steps_since_growth, num_steps;
} ora_scaler;
void ora_scaler_init(ora_scaler* s, float initial_scale, float growth_factor,
                     float backoff_factor, int64_t growth_interval,
                     float min_scale, float max_scale);
void ora_scaler_step(ora_scaler* s);
void ora_scaler_backoff(ora_scaler* s);

/* ---- unscale / finite check / norm / clip ------------------------------- */
void ora_unscale(int dtype, const void* g, int64_t n, float scale, void* out);
int64_t ora_count_nonfinite(int dtype, const void* g, int64_t n);
void ora_upcast(int dtype, const void* g, int64_t n, float* out);
double ora_sumsq_f32(const float* g, int64_t n);
float ora_clip_coef(float norm, float max_norm);
float ora_global_norm_clip(float** grads, const int64_t* numels, int ntensors,
                           float max_norm);

/* ---- optimizers (sgd.mojo, adam.mojo, adamw.mojo) ----------------------- */
void ora_sgd_step_f32(const float* p, const float* g, const float* vel,
                      int64_t n, double lr, double momentum, double wd,
                      float* out_p, float* out_vel);
void ora_sgd_step_f64(const double* p, const double* g, const double* vel,
                      int64_t n, double lr, double momentum, double wd,
                      double* out_p, double* out_vel);
void ora_adam_step_f32(const float* p, const float* g, const float* m,
                       const float* v, int64_t n, int64_t t, double lr,
                       double b1, double b2, double eps, double wd,
                       float* out_p, float* out_m, float* out_v);
void ora_adam_step_f64(const double* p, const double* g, const double* m,
                       const double* v, int64_t n, int64_t t, double lr,
                       double b1, double b2, double eps, double wd,
                       double* out_p, double* out_m, double* out_v);
void ora_adamw_step_f32(const float* p, const float* g, const float* m,
                        const float* v, int64_t n, int64_t t, double lr,
                        double b1, double b2, double eps, double wd,
                        float* out_p, float* out_m, float* out_v);
void ora_adamw_step_f64(const double* p, const double* g, const double* m,
                        const double* v, int64_t n, int64_t t, double lr,
                        double b1, double b2, double eps, double wd,
                        double* out_p, double* out_m, double* out_v);

/* lion.mojo:36-104, rmsprop.mojo:30-175 (pow(e, 2.0) restated as the
 * correctly rounded e*e), adagrad.mojo:30-120 */
void ora_lion_step_f32(const float* p, const float* g, const float* m, int64_t n, double lr, double b1,
                       double b2, double wd, float* out_p, float* out_m);
void ora_lion_step_f64(const double* p, const double* g, const double* m, int64_t n, double lr, double b1,
                       double b2, double wd, double* out_p, double* out_m);
void ora_rmsprop_step_f32(const float* p, const float* g, const float* sq, const float* buf, int64_t n,
                          double lr, double alpha, double eps, double wd, double momentum, float* out_p,
                          float* out_sq, float* out_buf);
void ora_rmsprop_step_f64(const double* p, const double* g, const double* sq, const double* buf, int64_t n,
                          double lr, double alpha, double eps, double wd, double momentum, double* out_p,
                          double* out_sq, double* out_buf);
void ora_adagrad_step_f32(const float* p, const float* g, const float* acc, int64_t n, double lr, double eps,
                          double wd, float* out_p, float* out_acc);
void ora_adagrad_step_f64(const double* p, const double* g, const double* acc, int64_t n, double lr,
                          double eps, double wd, double* out_p, double* out_acc);

/* ---- FP4 singles: one value with its own scale (MXFP4/NVFP4.from_float32,
 * from_float32_stochastic, to_float32; mxfp4.mojo:303-491, nvfp4.mojo:
 * 290-481).  kind ORA_Q_MXFP4 or ORA_Q_NVFP4; stochastic 0 gives
 * from_float32, else from_float32_stochastic with the given seed. */
void ora_fp4_single_encode(int kind, float x, int stochastic, uint64_t seed, uint8_t* value, uint8_t* scale);
float ora_fp4_single_decode(int kind, uint8_t value, uint8_t scale);

/* ---- the fused step (call stack B of the reference) --------------------- */
typedef struct {
  int64_t numel;
  int32_t grad_dtype;
  int32_t quant;
  float* master; /* in/out */
  float* s1;     /* velocity (SGD), m (Adam/AdamW/Lion), square_avg (RMSprop),
                    accumulator (Adagrad); may be NULL for SGD mu=0 */
  float* s2;     /* v (Adam/AdamW), momentum buffer (RMSprop with momentum) */
  const void* grad;
  uint8_t* qout;  /* ora_quant_bytes(quant, numel) bytes, or NULL */
  float* qscale;  /* per-tensor scale out, or NULL */
} ora_tensor;

typedef struct {
  int32_t optimizer;
  double lr, momentum, beta1, beta2, epsilon, weight_decay;
  int32_t use_scaler;
  int32_t clip_enabled;
  float max_norm;
  double alpha; /* RMSprop smoothing constant */
} ora_cfg;

typedef struct {
  int32_t skipped;
  int32_t clipped;
  int64_t nonfinite;
  double sumsq;
  float norm;
  float coef;
  float scale_used;
  float scale_next;
  int64_t step_count;
  int64_t overflow_count;
} ora_result;

int ora_fused_step(ora_tensor* ts, int nt, const ora_cfg* cfg, ora_scaler* sc,
                   int64_t* step_count, int64_t* overflow_count, int64_t t,
                   ora_result* res);

/* threads used by the OpenMP loops (0 = OpenMP default) */
void ora_set_threads(int n);
int ora_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
