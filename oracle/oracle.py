"""numpy bindings for the C oracle (libody_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, always as the checker (or the timed CPU
reference), never as part of the product path.  See ody_oracle.h for what
each function restates.
"""
import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libody_oracle.so")
_lib = None

F32, F16, BF16 = 0, 1, 2
SGD, ADAM, ADAMW, LION, RMSPROP, ADAGRAD = 0, 1, 2, 3, 4, 5
(Q_NONE, Q_FP16, Q_BF16, Q_FP8_E4M3, Q_FP8_E5M2, Q_FP8_E4M3_TENSOR, Q_MXFP4, Q_NVFP4, Q_NVFP4_TENSOR,
 Q_MXFP4_OCP) = range(10)

_p = C.c_void_p
_i64 = C.c_int64


class Scaler(C.Structure):
    _fields_ = [("scale", C.c_float), ("growth_factor", C.c_float), ("backoff_factor", C.c_float),
                ("min_scale", C.c_float), ("max_scale", C.c_float), ("growth_interval", _i64),
                ("steps_since_growth", _i64), ("num_steps", _i64)]


class Tensor(C.Structure):
    _fields_ = [("numel", _i64), ("grad_dtype", C.c_int32), ("quant", C.c_int32), ("master", _p),
                ("s1", _p), ("s2", _p), ("grad", _p), ("qout", _p), ("qscale", _p)]


class Cfg(C.Structure):
    _fields_ = [("optimizer", C.c_int32), ("lr", C.c_double), ("momentum", C.c_double),
                ("beta1", C.c_double), ("beta2", C.c_double), ("epsilon", C.c_double),
                ("weight_decay", C.c_double), ("use_scaler", C.c_int32), ("clip_enabled", C.c_int32),
                ("max_norm", C.c_float), ("alpha", C.c_double)]


class Result(C.Structure):
    _fields_ = [("skipped", C.c_int32), ("clipped", C.c_int32), ("nonfinite", _i64), ("sumsq", C.c_double),
                ("norm", C.c_float), ("coef", C.c_float), ("scale_used", C.c_float),
                ("scale_next", C.c_float), ("step_count", _i64), ("overflow_count", _i64)]


def build():
    """Compile libody_oracle.so from ody_oracle.c (gcc, no FMA contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sig = {
            "ora_f32_to_f16": (C.c_uint16, [C.c_float]), "ora_f16_to_f32": (C.c_float, [C.c_uint16]),
            "ora_f32_to_bf16": (C.c_uint16, [C.c_float]), "ora_bf16_to_f32": (C.c_float, [C.c_uint16]),
            "ora_f32_to_e4m3": (C.c_uint8, [C.c_float]), "ora_e4m3_to_f32": (C.c_float, [C.c_uint8]),
            "ora_f32_to_e5m2": (C.c_uint8, [C.c_float]), "ora_e5m2_to_f32": (C.c_float, [C.c_uint8]),
            "ora_e8m0_from_f32": (C.c_uint8, [C.c_float]), "ora_e8m0_to_f32": (C.c_float, [C.c_uint8]),
            "ora_e4m3_scale_from_f32": (C.c_uint8, [C.c_float]),
            "ora_fp4_from_f32": (C.c_uint8, [C.c_float, C.c_float]),
            "ora_fp4_to_f32": (C.c_float, [C.c_uint8, C.c_float]),
            "ora_mxfp4_block_encode": (None, [_p, _p]), "ora_mxfp4_block_decode": (None, [_p, _p]),
            "ora_nvfp4_block_encode": (None, [_p, _p]), "ora_nvfp4_block_decode": (None, [_p, _p]),
            "ora_quant_bytes": (_i64, [C.c_int, _i64]),
            "ora_quantize": (C.c_float, [C.c_int, _p, _i64, _p]),
            "ora_dequantize": (None, [C.c_int, _p, _i64, C.c_float, _p]),
            "ora_scaler_init": (None, [_p, C.c_float, C.c_float, C.c_float, _i64, C.c_float, C.c_float]),
            "ora_scaler_step": (None, [_p]), "ora_scaler_backoff": (None, [_p]),
            "ora_unscale": (None, [C.c_int, _p, _i64, C.c_float, _p]),
            "ora_count_nonfinite": (_i64, [C.c_int, _p, _i64]),
            "ora_upcast": (None, [C.c_int, _p, _i64, _p]),
            "ora_sumsq_f32": (C.c_double, [_p, _i64]),
            "ora_clip_coef": (C.c_float, [C.c_float, C.c_float]),
            "ora_global_norm_clip": (C.c_float, [_p, _p, C.c_int, C.c_float]),
            "ora_fused_step": (C.c_int, [_p, C.c_int, _p, _p, _p, _p, _i64, _p]),
            "ora_set_threads": (None, [C.c_int]), "ora_get_threads": (C.c_int, []),
            "ora_fp4_single_encode": (None, [C.c_int, C.c_float, C.c_int, C.c_uint64, _p, _p]),
            "ora_fp4_single_decode": (C.c_float, [C.c_int, C.c_uint8, C.c_uint8]),
        }
        for t in ("f32", "f64"):
            sig[f"ora_sgd_step_{t}"] = (None, [_p, _p, _p, _i64, C.c_double, C.c_double, C.c_double, _p, _p])
            for o in ("adam", "adamw"):
                sig[f"ora_{o}_step_{t}"] = (None, [_p, _p, _p, _p, _i64, _i64] + [C.c_double] * 5 + [_p, _p, _p])
            sig[f"ora_lion_step_{t}"] = (None, [_p, _p, _p, _i64] + [C.c_double] * 4 + [_p, _p])
            sig[f"ora_rmsprop_step_{t}"] = (None, [_p, _p, _p, _p, _i64] + [C.c_double] * 5 + [_p, _p, _p])
            sig[f"ora_adagrad_step_{t}"] = (None, [_p, _p, _p, _i64] + [C.c_double] * 3 + [_p, _p])
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def set_threads(n):
    lib().ora_set_threads(int(n))


def get_threads():
    return lib().ora_get_threads()


# ---- element casts (vectorised over numpy arrays via the C scalar fns) ----
def _vec(fn, arr, out_dtype):
    f = getattr(lib(), fn)
    flat = np.asarray(arr).ravel()
    return np.array([f(x) for x in flat.tolist()], dtype=out_dtype).reshape(np.shape(arr))


def f32_to_f16_bits(x):
    return _vec("ora_f32_to_f16", np.asarray(x, np.float32), np.uint16)


def f32_to_bf16_bits(x):
    return _vec("ora_f32_to_bf16", np.asarray(x, np.float32), np.uint16)


def f32_to_e4m3(x):
    return _vec("ora_f32_to_e4m3", np.asarray(x, np.float32), np.uint8)


def f32_to_e5m2(x):
    return _vec("ora_f32_to_e5m2", np.asarray(x, np.float32), np.uint8)


def e4m3_to_f32(b):
    return _vec("ora_e4m3_to_f32", np.asarray(b, np.uint8), np.float32)


def e5m2_to_f32(b):
    return _vec("ora_e5m2_to_f32", np.asarray(b, np.uint8), np.float32)


# ---- blocks and tensors ----
def mxfp4_block_encode(v):
    v = np.ascontiguousarray(v, np.float32)
    assert v.size == 32
    out = np.zeros(17, np.uint8)
    lib().ora_mxfp4_block_encode(_ptr(v), _ptr(out))
    return out


def mxfp4_block_decode(b):
    b = np.ascontiguousarray(b, np.uint8)
    out = np.zeros(32, np.float32)
    lib().ora_mxfp4_block_decode(_ptr(b), _ptr(out))
    return out


def nvfp4_block_encode(v):
    v = np.ascontiguousarray(v, np.float32)
    assert v.size == 16
    out = np.zeros(9, np.uint8)
    lib().ora_nvfp4_block_encode(_ptr(v), _ptr(out))
    return out


def nvfp4_block_decode(b):
    b = np.ascontiguousarray(b, np.uint8)
    out = np.zeros(16, np.float32)
    lib().ora_nvfp4_block_decode(_ptr(b), _ptr(out))
    return out


def quant_bytes(kind, n):
    return lib().ora_quant_bytes(kind, n)


def quantize(kind, x):
    """Returns (bytes, tensor_scale)."""
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(quant_bytes(kind, x.size), np.uint8)
    s = lib().ora_quantize(kind, _ptr(x), x.size, _ptr(out))
    return out, s


def dequantize(kind, q, n, tensor_scale=1.0):
    q = np.ascontiguousarray(q, np.uint8)
    out = np.zeros(n, np.float32)
    lib().ora_dequantize(kind, _ptr(q), n, tensor_scale, _ptr(out))
    return out


# ---- scaler ----
def scaler(initial_scale=65536.0, growth_factor=2.0, backoff_factor=0.5, growth_interval=2000,
           min_scale=1.0, max_scale=65536.0):
    s = Scaler()
    lib().ora_scaler_init(C.byref(s), initial_scale, growth_factor, backoff_factor, growth_interval,
                          min_scale, max_scale)
    return s


def scaler_step(s):
    lib().ora_scaler_step(C.byref(s))


def scaler_backoff(s):
    lib().ora_scaler_backoff(C.byref(s))


# ---- unscale / check / norm ----
def _gdtype(a):
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    raise TypeError("pass bf16 as (uint16 array, BF16)")


def unscale(g, scale, dtype=None):
    dtype = _gdtype(g) if dtype is None else dtype
    g = np.ascontiguousarray(g)
    out = np.empty_like(g)
    lib().ora_unscale(dtype, _ptr(g), g.size, scale, _ptr(out))
    return out


def count_nonfinite(g, dtype=None):
    dtype = _gdtype(g) if dtype is None else dtype
    g = np.ascontiguousarray(g)
    return lib().ora_count_nonfinite(dtype, _ptr(g), g.size)


def upcast(g, dtype=None):
    dtype = _gdtype(g) if dtype is None else dtype
    g = np.ascontiguousarray(g)
    out = np.empty(g.size, np.float32)
    lib().ora_upcast(dtype, _ptr(g), g.size, _ptr(out))
    return out


def sumsq_f32(g):
    g = np.ascontiguousarray(g, np.float32)
    return lib().ora_sumsq_f32(_ptr(g), g.size)


def global_norm_clip(grads, max_norm):
    """In place on a list of contiguous float32 arrays; returns the norm."""
    arr = (C.c_void_p * len(grads))(*[g.ctypes.data for g in grads])
    n = np.array([g.size for g in grads], np.int64)
    return lib().ora_global_norm_clip(arr, _ptr(n), len(grads), max_norm)


# ---- optimizers ----
def sgd_step(p, g, vel, lr, momentum=0.0, wd=0.0, f64=False):
    dt = np.float64 if f64 else np.float32
    p, g, vel = (np.ascontiguousarray(a, dt) for a in (p, g, vel))
    op, ov = np.empty_like(p), np.empty_like(vel)
    getattr(lib(), "ora_sgd_step_f64" if f64 else "ora_sgd_step_f32")(
        _ptr(p), _ptr(g), _ptr(vel), p.size, lr, momentum, wd, _ptr(op), _ptr(ov))
    return op, ov


def _adam(name, p, g, m, v, t, lr, b1, b2, eps, wd, f64):
    dt = np.float64 if f64 else np.float32
    p, g, m, v = (np.ascontiguousarray(a, dt) for a in (p, g, m, v))
    op, om, ov = np.empty_like(p), np.empty_like(m), np.empty_like(v)
    getattr(lib(), f"ora_{name}_step_{'f64' if f64 else 'f32'}")(
        _ptr(p), _ptr(g), _ptr(m), _ptr(v), p.size, t, lr, b1, b2, eps, wd, _ptr(op), _ptr(om), _ptr(ov))
    return op, om, ov


def adam_step(p, g, m, v, t, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, f64=False):
    return _adam("adam", p, g, m, v, t, lr, b1, b2, eps, wd, f64)


def adamw_step(p, g, m, v, t, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, f64=False):
    return _adam("adamw", p, g, m, v, t, lr, b1, b2, eps, wd, f64)


def lion_step(p, g, m, lr, b1=0.9, b2=0.99, wd=0.0, f64=False):
    dt = np.float64 if f64 else np.float32
    p, g, m = (np.ascontiguousarray(a, dt) for a in (p, g, m))
    op, om = np.empty_like(p), np.empty_like(m)
    getattr(lib(), f"ora_lion_step_{'f64' if f64 else 'f32'}")(
        _ptr(p), _ptr(g), _ptr(m), p.size, lr, b1, b2, wd, _ptr(op), _ptr(om))
    return op, om


def rmsprop_step(p, g, sq, lr, alpha=0.99, eps=1e-8, wd=0.0, momentum=0.0, buf=None, f64=False):
    dt = np.float64 if f64 else np.float32
    p, g, sq = (np.ascontiguousarray(a, dt) for a in (p, g, sq))
    bufa = np.ascontiguousarray(buf, dt) if buf is not None else None
    op, osq = np.empty_like(p), np.empty_like(sq)
    ob = np.zeros_like(p) if momentum > 0.0 else None
    getattr(lib(), f"ora_rmsprop_step_{'f64' if f64 else 'f32'}")(
        _ptr(p), _ptr(g), _ptr(sq), _ptr(bufa) if bufa is not None else None, p.size, lr, alpha, eps, wd,
        momentum, _ptr(op), _ptr(osq), _ptr(ob) if ob is not None else None)
    return op, osq, ob


def adagrad_step(p, g, acc, lr, eps=1e-10, wd=0.0, f64=False):
    dt = np.float64 if f64 else np.float32
    p, g, acc = (np.ascontiguousarray(a, dt) for a in (p, g, acc))
    op, oa = np.empty_like(p), np.empty_like(acc)
    getattr(lib(), f"ora_adagrad_step_{'f64' if f64 else 'f32'}")(
        _ptr(p), _ptr(g), _ptr(acc), p.size, lr, eps, wd, _ptr(op), _ptr(oa))
    return op, oa


def fp4_single_encode(kind, x, seeds=None):
    """(values, scales) of MXFP4/NVFP4.from_float32[_stochastic] per element."""
    x = np.ascontiguousarray(x, np.float32).ravel()
    vals, scs = np.zeros(x.size, np.uint8), np.zeros(x.size, np.uint8)
    v, sc = C.c_uint8(), C.c_uint8()
    f = lib().ora_fp4_single_encode
    for i in range(x.size):
        f(kind, float(x[i]), 0 if seeds is None else 1, 0 if seeds is None else int(seeds[i]), C.byref(v),
          C.byref(sc))
        vals[i], scs[i] = v.value, sc.value
    return vals, scs


def fp4_single_decode(kind, values, scales):
    f = lib().ora_fp4_single_decode
    return np.array([f(kind, int(a), int(b)) for a, b in zip(values, scales)], np.float32)


# ---- fused step over a model ----
class Model:
    """Host-side state of a whole model for ora_fused_step.

    tensors: list of dicts {numel, grad_dtype, quant}; master/s1/s2 float32
    arrays are owned here and updated in place by step()."""

    def __init__(self, specs, optimizer, lr, momentum=0.0, beta1=0.9, beta2=0.999, epsilon=1e-8,
                 weight_decay=0.0, use_scaler=True, clip_enabled=False, max_norm=1.0,
                 scaler_kwargs=None, alpha=0.99):
        self.specs = specs
        self.cfg = Cfg(optimizer, lr, momentum, beta1, beta2, epsilon, weight_decay, int(use_scaler),
                       int(clip_enabled), max_norm, alpha)
        self.scaler = scaler(**(scaler_kwargs or {}))
        self.step_count = C.c_int64(0)
        self.overflow_count = C.c_int64(0)
        self.master = [np.zeros(s["numel"], np.float32) for s in specs]
        self.s1 = [np.zeros(s["numel"], np.float32) for s in specs]
        self.s2 = [np.zeros(s["numel"], np.float32) for s in specs]
        self.qout = [np.zeros(max(quant_bytes(s["quant"], s["numel"]), 1), np.uint8) for s in specs]
        self.qscale = [np.ones(1, np.float32) for _ in specs]

    def step(self, grads, t):
        """grads: list of arrays (float32, float16, or uint16 holding bf16 bits)."""
        arr = (Tensor * len(self.specs))()
        keep = []
        for i, s in enumerate(self.specs):
            g = np.ascontiguousarray(grads[i])
            keep.append(g)
            arr[i] = Tensor(s["numel"], s["grad_dtype"], s["quant"], self.master[i].ctypes.data,
                            self.s1[i].ctypes.data, self.s2[i].ctypes.data, g.ctypes.data,
                            self.qout[i].ctypes.data, self.qscale[i].ctypes.data)
        res = Result()
        rc = lib().ora_fused_step(arr, len(self.specs), C.byref(self.cfg), C.byref(self.scaler),
                                  C.byref(self.step_count), C.byref(self.overflow_count), t,
                                  C.byref(res))
        if rc != 0:
            raise ValueError("Timestep t must be positive (starts at 1)")
        return res
