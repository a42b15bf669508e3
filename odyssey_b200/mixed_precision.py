"""Mirror of src/odyssey/training/mixed_precision.mojo over libodyssey_mp.so.

Same names, argument meaning and error texts as the reference.  Tensors are
numpy arrays (host) or torch tensors (host or CUDA; bfloat16 allowed);
bfloat16 numpy data is passed as uint16 with ``dtype='bfloat16'``.  All
element work runs in the CUDA library; the scaler's scalar state machine is
plain host arithmetic in float32, as in the reference.
"""
import ctypes as C

import numpy as np

from . import _lib as L
from .gradient_clipping import clip_gradients_by_global_norm


def _f32(x):
    return float(np.float32(x))


class GradientScaler:
    """GradientScaler (mixed_precision.mojo:45-237)."""

    def __init__(self, initial_scale=65536.0, growth_factor=2.0, backoff_factor=0.5,
                 growth_interval=2000, min_scale=1.0, max_scale=65536.0):
        self.scale = _f32(initial_scale)
        self.growth_factor = _f32(growth_factor)
        self.backoff_factor = _f32(backoff_factor)
        self.growth_interval = int(growth_interval)
        self._steps_since_growth = 0
        self._num_steps = 0
        self.min_scale = _f32(min_scale)
        self.max_scale = _f32(max_scale)

    def scale_loss(self, loss):
        """loss * full(shape, F64(scale), loss.dtype) (mixed_precision.mojo:124-152)."""
        if L.numel(loss) == 0:
            raise L.OdysseyError("Cannot scale empty loss tensor", L.ERR_SHAPE)
        if self.scale <= 0.0:
            raise L.OdysseyError("Scale factor must be positive, got: " + str(self.scale), L.ERR_ARG)
        if L.is_torch(loss):
            return loss * loss.new_full(loss.shape, self.scale)
        a = np.asarray(loss)
        return a * a.dtype.type(self.scale)

    def unscale_gradients(self, gradients, dtype=None):
        """gradients / full(shape, F64(scale), dtype) (mixed_precision.mojo:154-182)."""
        if L.numel(gradients) == 0:
            raise L.OdysseyError("Cannot unscale empty gradient tensor", L.ERR_SHAPE)
        if self.scale == 0.0:
            raise L.OdysseyError("Cannot unscale with zero scale factor", L.ERR_ARG)
        g = L.contiguous(gradients)
        out = L.empty_like(g)
        L.check(L.lib().ody_unscale(L.ptr(g), L.dtype_code(g, dtype), L.numel(g), self.scale, L.ptr(out)))
        return out

    def step(self):
        """mixed_precision.mojo:184-205 (float32 arithmetic)."""
        self._num_steps += 1
        self._steps_since_growth += 1
        if self._steps_since_growth >= self.growth_interval:
            new_scale = _f32(np.float32(self.scale) * np.float32(self.growth_factor))
            self.scale = self.max_scale if new_scale > self.max_scale else new_scale
            self._steps_since_growth = 0

    def backoff(self):
        """mixed_precision.mojo:207-221."""
        new_scale = _f32(np.float32(self.scale) * np.float32(self.backoff_factor))
        if new_scale >= self.min_scale:
            self.scale = new_scale
        self._steps_since_growth = 0

    def get_scale(self):
        return self.scale

    def get_num_steps(self):
        return self._num_steps


def convert_to_fp32_master(params, dtype=None):
    """FP32 copy of parameters (mixed_precision.mojo:240-296)."""
    if L.numel(params) == 0:
        raise L.OdysseyError("Cannot convert empty parameter tensor", L.ERR_SHAPE)
    p = L.contiguous(params)
    out = L.empty_like(p, "float32")
    L.check(L.lib().ody_to_fp32(L.ptr(p), L.dtype_code(p, dtype), L.numel(p), L.ptr(out)))
    return out


def update_model_from_master(model_params, master_params, dtype=None):
    """Cast FP32 master weights into the model tensor, in place
    (mixed_precision.mojo:299-354)."""
    if L.numel(model_params) == 0 or L.numel(master_params) == 0:
        raise L.OdysseyError("Cannot update from empty tensors", L.ERR_SHAPE)
    if L.numel(model_params) != L.numel(master_params):
        raise L.OdysseyError("Parameter and master weight sizes must match", L.ERR_SHAPE)
    if L.dtype_code(master_params) != L.F32:
        raise L.OdysseyError("Master params must be Float32, got: " + str(master_params.dtype), L.ERR_DTYPE)
    code = L.dtype_code(model_params, dtype)
    m = L.contiguous(master_params)
    if code == L.F32:
        if L.is_torch(model_params):
            model_params.copy_(m.reshape(model_params.shape))
        else:
            np.copyto(model_params, np.asarray(m).reshape(np.shape(model_params)))
        return
    kind = L.Q_FP16 if code == L.F16 else L.Q_BF16
    L.check(L.lib().ody_quantize(kind, L.ptr(m), L.F32, L.numel(m), L.ptr(model_params), None))


def check_gradients_finite(gradients, dtype=None):
    """True when no NaN/Inf (mixed_precision.mojo:357-381)."""
    g = L.contiguous(gradients)
    fin = C.c_int32(0)
    L.check(L.lib().ody_check_finite(L.ptr(g), L.dtype_code(g, dtype), L.numel(g), C.byref(fin)))
    return bool(fin.value)


def clip_gradients_by_norm(gradients, max_norm):
    """Clip one float32 gradient tensor to max_norm (mixed_precision.mojo:384-433).

    The reference sums g*g serially with the accumulator rounded to the
    tensor dtype after every add; here the sum is accumulated in float64 on
    the GPU and the coefficient is clip_gradients_by_global_norm's, so the
    result agrees with the reference to float32 rounding (the reference's
    own tests use tolerance 1e-5)."""
    if max_norm <= 0.0:
        raise L.OdysseyError("max_norm must be positive, got: " + str(max_norm), L.ERR_ARG)
    if L.numel(gradients) == 0:
        return gradients
    g = L.contiguous(gradients).copy() if not L.is_torch(gradients) else gradients.contiguous().clone()
    clip_gradients_by_global_norm([g], max_norm)
    return g
