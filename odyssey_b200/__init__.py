"""odyssey_b200 -- B200-native (sm_100a) mixed-precision parameter-update path
of Odyssey, behind the C ABI of libodyssey_mp.so (include/odyssey_mp.h).

Python mirror of the reference's training / quant-type API:
GradientScaler, PrecisionConfig, convert_to_fp32_master,
update_model_from_master, check_gradients_finite, clip_gradients_by_norm,
clip_gradients_by_global_norm, sgd_step / adam_step / adamw_step /
lion_step / rmsprop_step / adagrad_step,
to_/from_{fp8,bf8,mxfp4,nvfp4}, plus the fused MixedPrecisionStep.
"""
from ._lib import LIB_PATH, OdysseyError, lib  # noqa: F401
from .fused import MixedPrecisionStep, nccl_unique_id, plan_shards  # noqa: F401
from .gradient_clipping import (clip_global_norm, clip_grad_global_norm_,  # noqa: F401
                                clip_gradients_by_global_norm, compute_gradient_norm_list)
from .mixed_precision import (GradientScaler, check_gradients_finite, clip_gradients_by_norm,  # noqa: F401
                              convert_to_fp32_master, update_model_from_master)
from .optimizers import (adagrad_step, adagrad_step_simple, adam_step, adamw_step,  # noqa: F401
                         adamw_step_simple, init_adagrad_state, init_adam_state, init_adamw_state,
                         init_lion_state, init_rmsprop_state, init_sgd_state, lion_step, lion_step_simple,
                         rmsprop_step, rmsprop_step_simple, sgd_step)
from .precision_config import PrecisionConfig, PrecisionMode  # noqa: F401
from .quant import (MXFP4, NVFP4, QuantizedTensor, dequantize, from_bf8, from_fp8, from_mxfp4, from_nvfp4,  # noqa: F401
                    quantize, to_bf8, to_fp8, to_fp8_tensor_scaled, to_mxfp4, to_mxfp4_ocp, to_nvfp4,
                    to_nvfp4_tensor_scaled)
