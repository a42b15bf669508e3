"""Mirror of src/odyssey/training/precision_config.mojo:68-591."""
from . import _lib as L
from .mixed_precision import GradientScaler, check_gradients_finite, clip_gradients_by_norm, \
    convert_to_fp32_master


class PrecisionMode:
    """precision_config.mojo:68-130."""
    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    FP8 = "fp8"


class PrecisionConfig:
    """precision_config.mojo:133-591: mode, dtypes, an owned GradientScaler
    and the overflow / step counters."""

    def __init__(self, mode, compute_dtype, storage_dtype, use_gradient_scaler=True, initial_scale=65536.0):
        self.mode = mode
        self.compute_dtype = compute_dtype
        self.storage_dtype = storage_dtype
        self.master_dtype = "float32"
        self.use_gradient_scaler = use_gradient_scaler
        self.scaler = GradientScaler(initial_scale=initial_scale)
        self._overflow_count = 0
        self._step_count = 0

    @staticmethod
    def fp32():
        return PrecisionConfig(PrecisionMode.FP32, "float32", "float32", use_gradient_scaler=False)

    @staticmethod
    def fp16(initial_scale=65536.0):
        return PrecisionConfig(PrecisionMode.FP16, "float16", "float16", True, initial_scale)

    @staticmethod
    def bf16(initial_scale=65536.0):
        return PrecisionConfig(PrecisionMode.BF16, "bfloat16", "bfloat16", True, initial_scale)

    @staticmethod
    def fp8(initial_scale=65536.0):
        """FP8 mode computes and stores in FP16 (precision_config.mojo:284-327)."""
        return PrecisionConfig(PrecisionMode.FP8, "float16", "float16", True, initial_scale)

    @staticmethod
    def from_string(precision_str):
        table = {"fp32": PrecisionConfig.fp32, "fp16": PrecisionConfig.fp16, "bf16": PrecisionConfig.bf16,
                 "fp8": PrecisionConfig.fp8}
        if precision_str not in table:
            raise L.OdysseyError("Unknown precision: " + precision_str + ". Use fp32, fp16, bf16, or fp8.",
                                 L.ERR_ARG)
        return table[precision_str]()

    def cast_to_master(self, tensor, dtype=None):
        return convert_to_fp32_master(tensor, dtype)

    def scale_loss(self, loss):
        return loss if not self.use_gradient_scaler else self.scaler.scale_loss(loss)

    def unscale_gradients(self, gradients, dtype=None):
        return gradients if not self.use_gradient_scaler else self.scaler.unscale_gradients(gradients, dtype)

    def check_gradients(self, gradients, dtype=None):
        return check_gradients_finite(gradients, dtype)

    def step(self, grads_valid):
        """precision_config.mojo:455-473."""
        self._step_count += 1
        if not self.use_gradient_scaler:
            return
        if grads_valid:
            self.scaler.step()
        else:
            self.scaler.backoff()
            self._overflow_count += 1

    def get_scale(self):
        return self.scaler.get_scale()

    def get_overflow_count(self):
        return self._overflow_count

    def get_step_count(self):
        return self._step_count

    def needs_master_weights(self):
        return self.mode != PrecisionMode.FP32

    def clip_gradients(self, gradients, max_norm):
        return clip_gradients_by_norm(gradients, max_norm)
