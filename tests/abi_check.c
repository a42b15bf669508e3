/* A plain C caller of libodyssey_mp.so (the way a native binding would use
 * include/odyssey_mp.h): host-only entry points and their error paths, so
 * it runs without a GPU.  Built and run by tests/test_abi.py. */
#include <stdio.h>
#include <string.h>

#include "odyssey_mp.h"

#define CHECK(c)                                                        \
  do {                                                                  \
    if (!(c)) {                                                         \
      fprintf(stderr, "FAIL %s:%d: %s (%s)\n", __FILE__, __LINE__, #c,  \
              ody_last_error(NULL));                                    \
      return 1;                                                         \
    }                                                                   \
  } while (0)

int main(void) {
  CHECK(ody_abi_version() > 0);
  ody_config cfg;
  ody_config_default(&cfg);
  CHECK(cfg.optimizer == ODY_ADAMW && cfg.initial_scale == 65536.0f && cfg.growth_interval == 2000);
  CHECK(cfg.max_scale == 65536.0f && cfg.alpha == 0.99);
  CHECK(sizeof(ody_config) == 128);

  /* AoS block sizes (tensor_dtype_conv.mojo:281-366) */
  CHECK(ody_quant_bytes(ODY_Q_MXFP4, 33) == 2 * 17);
  CHECK(ody_quant_bytes(ODY_Q_NVFP4, 16) == 9);
  CHECK(ody_quant_bytes(ODY_Q_FP16, 5) == 10);
  CHECK(ody_quant_bytes(ODY_Q_FP8_E4M3, 7) == 7);

  /* ZeRO-1 plan: contiguous runs of whole tensors in rank order */
  int64_t numels[6] = {100, 200, 300, 400, 500, 600};
  int32_t owner[6];
  CHECK(ody_plan_shards(numels, 6, 3, owner) == ODY_OK);
  CHECK(owner[0] == 0 && owner[5] == 2);
  for (int i = 1; i < 6; i++) CHECK(owner[i] >= owner[i - 1] && owner[i] - owner[i - 1] <= 1);

  /* configuration errors carry the reference's messages */
  ody_ctx* ctx = NULL;
  cfg.optimizer = 99;
  CHECK(ody_ctx_create(&ctx, &cfg) == ODY_ERR_ARG);
  CHECK(strstr(ody_last_error(NULL), "unknown optimizer") != NULL);
  ody_config_default(&cfg);
  cfg.initial_scale = 0.0f;
  CHECK(ody_ctx_create(&ctx, &cfg) == ODY_ERR_ARG);
  CHECK(strstr(ody_last_error(NULL), "Cannot unscale with zero scale factor") != NULL);

  /* a context before finalize: registration works, steps are refused */
  ody_config_default(&cfg);
  cfg.optimizer = ODY_LION;
  CHECK(ody_ctx_create(&ctx, &cfg) == ODY_OK && ctx != NULL);
  int32_t idx = -1;
  CHECK(ody_ctx_add_tensor(ctx, 1000, ODY_BF16, ODY_Q_NVFP4_TENSOR, &idx) == ODY_OK && idx == 0);
  CHECK(ody_ctx_add_tensor(ctx, 64, ODY_BF16, ODY_Q_MXFP4, &idx) == ODY_OK && idx == 1);
  ody_step_result res;
  CHECK(ody_step(ctx, 1, &res) == ODY_ERR_STATE);
  CHECK(strstr(ody_last_error(ctx), "not finalized") != NULL);
  ody_ctx_destroy(ctx);

  /* argument checks that come before any device work */
  float x[4] = {1, 2, 3, 4};
  unsigned char v[4], s[4];
  CHECK(ody_fp4_single_encode(ODY_Q_FP16, x, 4, NULL, v, s) == ODY_ERR_ARG);
  CHECK(ody_quantize(ODY_Q_MXFP4, x, ODY_F32, 0, v, NULL) == ODY_ERR_SHAPE);
  CHECK(ody_quantize(42, x, ODY_F32, 4, v, NULL) == ODY_ERR_ARG);
  printf("ok\n");
  return 0;
}
