"""Mirror of src/odyssey/training/optimizers/{sgd,adam,adamw,lion,rmsprop,
adagrad}.mojo over libodyssey_mp.so: pure functional steps returning new
tensors."""
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


def lion_step(params, gradients, momentum, learning_rate, beta1=0.9, beta2=0.99, weight_decay=0.0):
    """lion.mojo:36-104 -> (new_params, new_momentum)."""
    if tuple(np.shape(params)) != tuple(np.shape(gradients)):
        raise L.OdysseyError("lion_step: params and gradients must have the same shape", L.ERR_SHAPE)
    if momentum is None or tuple(np.shape(params)) != tuple(np.shape(momentum)):
        raise L.OdysseyError("lion_step: params and momentum must have the same shape", L.ERR_SHAPE)
    if L.dtype_code(params) != L.dtype_code(gradients):
        raise L.OdysseyError("lion_step: params and gradients must have the same dtype", L.ERR_DTYPE)
    _check_pair(params, gradients)
    p, g, m = (L.contiguous(a) for a in (params, gradients, momentum))
    op, om = L.empty_like(p), L.empty_like(p)
    L.check(L.lib().ody_lion_step(L.ptr(p), L.ptr(g), L.ptr(m), L.numel(p), learning_rate, beta1, beta2,
                                  weight_decay, L.ptr(op), L.ptr(om)))
    return op, om


def lion_step_simple(params, gradients, momentum, learning_rate):
    """lion.mojo:109-142."""
    return lion_step(params, gradients, momentum, learning_rate, 0.9, 0.99, 0.0)


def rmsprop_step(params, gradients, square_avg, t, learning_rate, alpha=0.99, epsilon=1e-8, weight_decay=0.0,
                 momentum=0.0, buf=None):
    """rmsprop.mojo:30-175 -> (new_params, new_square_avg, new_buf); new_buf is
    the given buffer (or an empty one) when momentum is 0."""
    _check_pair(params, gradients)
    if square_avg is None or L.numel(square_avg) == 0:
        raise L.OdysseyError("square_avg must be initialized (use zeros_like(params))", L.ERR_ARG)
    if t <= 0:
        raise L.OdysseyError("Timestep t must be positive (starts at 1)", L.ERR_ARG)
    p, g, sq = (L.contiguous(a) for a in (params, gradients, square_avg))
    b = L.contiguous(buf) if (momentum > 0.0 and buf is not None and L.numel(buf)) else None
    op, osq = L.empty_like(p), L.empty_like(p)
    ob = L.empty_like(p) if momentum > 0.0 else None
    L.check(L.lib().ody_rmsprop_step(L.ptr(p), L.ptr(g), L.ptr(sq), L.ptr(b), L.numel(p), t, learning_rate,
                                     alpha, epsilon, weight_decay, momentum, L.ptr(op), L.ptr(osq), L.ptr(ob)))
    if ob is None:
        ob = buf if buf is not None else np.zeros(0, np.float32)
    return op, osq, ob


def rmsprop_step_simple(params, gradients, square_avg, learning_rate, alpha=0.99, epsilon=1e-8):
    """rmsprop.mojo:178-231."""
    op, osq, _ = rmsprop_step(params, gradients, square_avg, 1, learning_rate, alpha, epsilon)
    return op, osq


def adagrad_step(params, gradients, accum, learning_rate, epsilon=1e-10, weight_decay=0.0):
    """adagrad.mojo:30-113 -> (new_params, new_accum)."""
    _check_pair(params, gradients)
    if accum is None or L.numel(accum) == 0:
        raise L.OdysseyError("accumulator must be initialized (use zeros_like(params))", L.ERR_ARG)
    p, g, a = (L.contiguous(x) for x in (params, gradients, accum))
    op, oa = L.empty_like(p), L.empty_like(p)
    L.check(L.lib().ody_adagrad_step(L.ptr(p), L.ptr(g), L.ptr(a), L.numel(p), learning_rate, epsilon,
                                     weight_decay, L.ptr(op), L.ptr(oa)))
    return op, oa


def adagrad_step_simple(params, gradients, accum, learning_rate):
    """adagrad.mojo:116-161."""
    return adagrad_step(params, gradients, accum, learning_rate, 1e-10, 0.0)


def init_lion_state(params_list, force_f64=False):
    """lion.mojo:145-176: one zero momentum per parameter."""
    return [[_zeros_like(p, force_f64)] for p in params_list]


def init_rmsprop_state(params_list, force_f64=False):
    """rmsprop.mojo:234-265: zero square_avg and momentum buffer per parameter."""
    return [[_zeros_like(p, force_f64), _zeros_like(p, force_f64)] for p in params_list]


def init_adagrad_state(params_list, force_f64=False):
    """adagrad.mojo:164-197: one zero accumulator per parameter."""
    return [[_zeros_like(p, force_f64)] for p in params_list]
