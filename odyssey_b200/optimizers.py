"""Mirror of src/odyssey/training/optimizers/{sgd,adam,adamw}.mojo over
libodyssey_mp.so: pure functional steps returning new tensors."""
import numpy as np

from . import _lib as L


def _check_pair(params, gradients):
    if tuple(np.shape(params)) != tuple(np.shape(gradients)):
        raise L.OdysseyError("Parameters and gradients must have the same shape", L.ERR_SHAPE)
    if L.dtype_code(params) != L.dtype_code(gradients):
        raise L.OdysseyError("Parameters and gradients must have the same dtype", L.ERR_DTYPE)
    if L.dtype_code(params) != L.F32:
        raise L.OdysseyError("the CUDA optimizers take float32 parameters", L.ERR_DTYPE)


def sgd_step(params, gradients, velocity, learning_rate, momentum=0.0, weight_decay=0.0):
    """sgd.mojo:27-121 -> (new_params, new_velocity)."""
    _check_pair(params, gradients)
    if momentum > 0.0 and (velocity is None or L.numel(velocity) == 0):
        raise L.OdysseyError("Velocity buffer required when using momentum (use zeros_like(params))", L.ERR_ARG)
    p, g = L.contiguous(params), L.contiguous(gradients)
    v = L.contiguous(velocity) if velocity is not None and L.numel(velocity) else None
    op = L.empty_like(p)
    ov = L.empty_like(p) if v is not None else None
    L.check(L.lib().ody_sgd_step(L.ptr(p), L.ptr(g), L.ptr(v), L.numel(p), learning_rate, momentum,
                                 weight_decay, L.ptr(op), L.ptr(ov)))
    return op, (ov if ov is not None else velocity)


def _adam(fn, params, gradients, m, v, t, learning_rate, beta1, beta2, epsilon, weight_decay):
    _check_pair(params, gradients)
    if m is None or v is None or L.numel(m) == 0 or L.numel(v) == 0:
        raise L.OdysseyError("Moment buffers (m and v) must be initialized (use zeros_like(params))", L.ERR_ARG)
    if t <= 0:
        raise L.OdysseyError("Timestep t must be positive (starts at 1)", L.ERR_ARG)
    p, g, mm, vv = (L.contiguous(a) for a in (params, gradients, m, v))
    op, om, ov = L.empty_like(p), L.empty_like(p), L.empty_like(p)
    L.check(getattr(L.lib(), fn)(L.ptr(p), L.ptr(g), L.ptr(mm), L.ptr(vv), L.numel(p), t, learning_rate,
                                 beta1, beta2, epsilon, weight_decay, L.ptr(op), L.ptr(om), L.ptr(ov)))
    return op, om, ov


def adam_step(params, gradients, m, v, t, learning_rate, beta1=0.9, beta2=0.999, epsilon=1e-8,
              weight_decay=0.0):
    """adam.mojo:42-166 -> (new_params, new_m, new_v)."""
    return _adam("ody_adam_step", params, gradients, m, v, t, learning_rate, beta1, beta2, epsilon,
                 weight_decay)


def adamw_step(params, gradients, m, v, t, learning_rate, beta1=0.9, beta2=0.999, epsilon=1e-8,
               weight_decay=0.01):
    """adamw.mojo:44-175 -> (new_params, new_m, new_v); decoupled decay on the
    post-update params without an lr factor."""
    return _adam("ody_adamw_step", params, gradients, m, v, t, learning_rate, beta1, beta2, epsilon,
                 weight_decay)


def adamw_step_simple(params, gradients, m, v, t, learning_rate):
    """adamw.mojo:178-239."""
    return adamw_step(params, gradients, m, v, t, learning_rate, 0.9, 0.999, 1e-8, 0.01)


def _zeros_like(p, force_f64=False):
    if L.is_torch(p):
        import torch
        return torch.zeros_like(p, dtype=torch.float64 if force_f64 else p.dtype)
    return np.zeros(np.shape(p), np.float64 if force_f64 else np.asarray(p).dtype)


def init_sgd_state(params_list, force_f64=False):
    """sgd.mojo:350-381: one zero velocity per parameter."""
    return [[_zeros_like(p, force_f64)] for p in params_list]


def init_adam_state(params_list, force_f64=False):
    """adam.mojo:231-262: zero m and v per parameter."""
    return [[_zeros_like(p, force_f64), _zeros_like(p, force_f64)] for p in params_list]


def init_adamw_state(params_list, force_f64=False):
    """adamw.mojo:242-273."""
    return init_adam_state(params_list, force_f64)
