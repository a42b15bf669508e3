"""ctypes binding of libodyssey_mp.so (include/odyssey_mp.h).

The CUDA library is the product: there is no CPU fallback.  If the shared
library is missing or fails to load, every call raises OdysseyError.
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ODYSSEY_MP_LIB") or os.path.join(_HERE, "libodyssey_mp.so")

OK = 0
ERR_ARG, ERR_SHAPE, ERR_DTYPE, ERR_CUDA, ERR_NCCL, ERR_COMM_TIMEOUT, ERR_DEVICE_BOUNDS, ERR_STATE = range(-1, -9, -1)
F32, F16, BF16 = 0, 1, 2
SGD, ADAM, ADAMW, LION, RMSPROP, ADAGRAD = 0, 1, 2, 3, 4, 5
(Q_NONE, Q_FP16, Q_BF16, Q_FP8_E4M3, Q_FP8_E5M2, Q_FP8_E4M3_TENSOR, Q_MXFP4, Q_NVFP4,
 Q_NVFP4_TENSOR, Q_MXFP4_OCP) = range(10)
BUF_MASTER, BUF_STATE1, BUF_STATE2, BUF_GRAD, BUF_DP_GRAD = range(5)

QUANT_NAMES = {
    "none": Q_NONE, "fp16": Q_FP16, "bf16": Q_BF16, "fp8": Q_FP8_E4M3, "fp8_e4m3": Q_FP8_E4M3,
    "bf8": Q_FP8_E5M2, "fp8_e5m2": Q_FP8_E5M2, "fp8_tensor": Q_FP8_E4M3_TENSOR, "mxfp4": Q_MXFP4,
    "nvfp4": Q_NVFP4, "nvfp4_tensor": Q_NVFP4_TENSOR, "mxfp4_ocp": Q_MXFP4_OCP,
}


class OdysseyError(RuntimeError):
    """A non-zero status of libodyssey_mp.so; the message is ody_last_error()."""

    def __init__(self, msg, code=ERR_ARG):
        super().__init__(msg)
        self.code = code


class Config(C.Structure):
    _fields_ = [
        ("optimizer", C.c_int32), ("device", C.c_int32), ("learning_rate", C.c_double),
        ("momentum", C.c_double), ("beta1", C.c_double), ("beta2", C.c_double), ("epsilon", C.c_double),
        ("weight_decay", C.c_double), ("use_gradient_scaler", C.c_int32), ("initial_scale", C.c_float),
        ("growth_factor", C.c_float), ("backoff_factor", C.c_float), ("growth_interval", C.c_int64),
        ("min_scale", C.c_float), ("max_scale", C.c_float), ("clip_enabled", C.c_int32),
        ("max_norm", C.c_float), ("comm_timeout_ms", C.c_int32), ("reserved0", C.c_int32),
        ("alpha", C.c_double), ("chunk_elems", C.c_int32), ("requant_placement", C.c_int32),
        ("reserved", C.c_int32 * 2),
    ]


class StepResult(C.Structure):
    _fields_ = [
        ("found_inf", C.c_int32), ("skipped", C.c_int32), ("clipped", C.c_int32), ("reserved0", C.c_int32),
        ("nonfinite_count", C.c_int64), ("sumsq", C.c_double), ("grad_norm", C.c_float),
        ("clip_coef", C.c_float), ("scale_used", C.c_float), ("scale_next", C.c_float),
        ("step_count", C.c_int64), ("overflow_count", C.c_int64), ("scaler_num_steps", C.c_int64),
        ("steps_since_growth", C.c_int64),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_ if not k.startswith("reserved")}


_p = C.c_void_p
_i32, _i64 = C.c_int32, C.c_int64
_SIGS = {
    "ody_abi_version": (C.c_int, []),
    "ody_last_error": (C.c_char_p, [_p]),
    "ody_config_default": (None, [_p]),
    "ody_quant_bytes": (_i64, [_i32, _i64]),
    "ody_ctx_create": (C.c_int, [_p, _p]),
    "ody_ctx_add_tensor": (C.c_int, [_p, _i64, _i32, _i32, _p]),
    "ody_ctx_finalize": (C.c_int, [_p, _i32, _i32, _p]),
    "ody_nccl_unique_id": (C.c_int, [_p]),
    "ody_plan_shards": (C.c_int, [_p, _i32, _i32, _p]),
    "ody_ctx_tensor_owner": (C.c_int, [_p, _i32, _p]),
    "ody_ctx_num_tensors": (C.c_int, [_p, _p]),
    "ody_upload": (C.c_int, [_p, _i32, _i32, _p, C.c_size_t]),
    "ody_upload_async": (C.c_int, [_p, _i32, _i32, _p, C.c_size_t]),
    "ody_download": (C.c_int, [_p, _i32, _i32, _p, C.c_size_t]),
    "ody_ctx_device_ptr": (C.c_int, [_p, _i32, _i32, _p]),
    "ody_ctx_stream": (C.c_int, [_p, _p]),
    "ody_step": (C.c_int, [_p, _i64, _p]),
    "ody_step_async": (C.c_int, [_p, _i64]),
    "ody_step_wait": (C.c_int, [_p, _p]),
    "ody_ctx_set_timing": (C.c_int, [_p, _i32]),
    "ody_ctx_pass_times": (C.c_int, [_p, _p, _p]),
    "ody_ctx_set_graph": (C.c_int, [_p, _i32]),
    "ody_ctx_set_grad_double_buffer": (C.c_int, [_p, _i32]),
    "ody_ctx_dp_attach": (C.c_int, [_p]),
    "ody_ctx_quant_layout": (C.c_int, [_p, _i32, _p, _p, _p]),
    "ody_ctx_gather_quant": (C.c_int, [_p, _p, _p]),
    "ody_get_quant": (C.c_int, [_p, _i32, _p, C.c_size_t, _p]),
    "ody_get_scaler": (C.c_int, [_p, _p, _p, _p, _p, _p]),
    "ody_set_scaler": (C.c_int, [_p, C.c_float, _i64, _i64, _i64, _i64]),
    "ody_ctx_export": (C.c_int, [_p, _p, _p]),
    "ody_ctx_import": (C.c_int, [_p, _p, C.c_size_t]),
    "ody_ctx_destroy": (None, [_p]),
    "ody_unscale": (C.c_int, [_p, _i32, _i64, C.c_float, _p]),
    "ody_check_finite": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_to_fp32": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_global_norm_clip": (C.c_int, [_p, _p, _i32, C.c_float, _p]),
    "ody_global_norm_clip_noalloc": (C.c_int, [_p, _p, _i32, C.c_float, _p]),
    "ody_sgd_step": (C.c_int, [_p, _p, _p, _i64, C.c_double, C.c_double, C.c_double, _p, _p]),
    "ody_adam_step": (C.c_int, [_p, _p, _p, _p, _i64, _i64] + [C.c_double] * 5 + [_p, _p, _p]),
    "ody_adamw_step": (C.c_int, [_p, _p, _p, _p, _i64, _i64] + [C.c_double] * 5 + [_p, _p, _p]),
    "ody_lion_step": (C.c_int, [_p, _p, _p, _i64] + [C.c_double] * 4 + [_p, _p]),
    "ody_clip_global_norm_variant": (C.c_int, [_p, _p, _i32, C.c_double, _i32, _p]),
    "ody_fp4_single_encode": (C.c_int, [_i32, _p, _i64, _p, _p, _p]),
    "ody_quantize_on_stream": (C.c_int, [_i32, _p, _i32, _i64, _p, _p, _p, _p]),
    "ody_dequantize_on_stream": (C.c_int, [_i32, _p, _i64, _p, _p, _p]),
    "ody_quant_mxfp4": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_dequant_mxfp4": (C.c_int, [_p, _i64, _p]),
    "ody_quant_nvfp4": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_dequant_nvfp4": (C.c_int, [_p, _i64, _p]),
    "ody_quant_fp8_e4m3": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_dequant_fp8_e4m3": (C.c_int, [_p, _i64, _p]),
    "ody_quant_fp8_e5m2": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_dequant_fp8_e5m2": (C.c_int, [_p, _i64, _p]),
    "ody_quant_fp16": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_dequant_fp16": (C.c_int, [_p, _i64, _p]),
    "ody_quant_bf16": (C.c_int, [_p, _i32, _i64, _p]),
    "ody_dequant_bf16": (C.c_int, [_p, _i64, _p]),
    "ody_fp4_single_decode": (C.c_int, [_i32, _p, _p, _i64, _p]),
    "ody_rmsprop_step": (C.c_int, [_p, _p, _p, _p, _i64, _i64] + [C.c_double] * 5 + [_p, _p, _p]),
    "ody_adagrad_step": (C.c_int, [_p, _p, _p, _i64] + [C.c_double] * 3 + [_p, _p]),
    "ody_quantize": (C.c_int, [_i32, _p, _i32, _i64, _p, _p]),
    "ody_dequantize": (C.c_int, [_i32, _p, _i64, C.c_float, _p]),
}
EXPORTED = tuple(_SIGS)

_lib = None


def lib():
    """The loaded library; raises OdysseyError if it cannot be loaded."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OdysseyError(f"{LIB_PATH} is missing: build it with `python -m odyssey_b200.build`",
                               ERR_STATE)
        try:
            L = C.CDLL(LIB_PATH)
        except OSError as e:
            raise OdysseyError(f"cannot load {LIB_PATH}: {e}", ERR_STATE) from e
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error(ctx=None):
    msg = lib().ody_last_error(ctx)
    return msg.decode() if msg else ""


def check(rc, ctx=None):
    if rc != OK:
        raise OdysseyError(last_error(ctx), rc)
    return rc


def default_config():
    cfg = Config()
    lib().ody_config_default(C.byref(cfg))
    return cfg


def quant_bytes(kind, n):
    return int(lib().ody_quant_bytes(kind, n))


# ---- buffers: numpy arrays (host) or torch tensors (host or CUDA) ----------
def _torch():
    try:
        import torch  # noqa: F401
        return torch
    except ImportError:
        return None


def is_torch(x):
    t = _torch()
    return t is not None and isinstance(x, t.Tensor)


def dtype_code(x, dtype=None):
    """F32/F16/BF16 code of an array; numpy bfloat16 data is passed as uint16
    with dtype='bfloat16'."""
    if dtype is not None:
        return {"float32": F32, "float16": F16, "bfloat16": BF16, F32: F32, F16: F16, BF16: BF16}[dtype]
    if is_torch(x):
        t = _torch()
        m = {t.float32: F32, t.float16: F16, t.bfloat16: BF16}
        if x.dtype not in m:
            raise OdysseyError(f"unsupported dtype {x.dtype}", ERR_DTYPE)
        return m[x.dtype]
    a = np.asarray(x)
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    raise OdysseyError(f"unsupported dtype {a.dtype} (pass bfloat16 as uint16 with dtype='bfloat16')",
                       ERR_DTYPE)


def ptr(x):
    """Address of a contiguous numpy array or torch tensor."""
    if x is None:
        return None
    if is_torch(x):
        if not x.is_contiguous():
            raise OdysseyError("tensor must be contiguous", ERR_ARG)
        return x.data_ptr()
    if not x.flags["C_CONTIGUOUS"]:
        raise OdysseyError("array must be C-contiguous", ERR_ARG)
    return x.ctypes.data


def numel(x):
    return x.numel() if is_torch(x) else int(np.asarray(x).size)


def empty_like(x, dtype=None, n=None):
    """A new buffer on the same side (host numpy / torch device) as x."""
    if is_torch(x):
        t = _torch()
        td = {None: x.dtype, "float32": t.float32, "uint8": t.uint8, "float16": t.float16,
              "bfloat16": t.bfloat16}[dtype]
        return t.empty(n if n is not None else x.shape, dtype=td, device=x.device)
    nd = {None: np.asarray(x).dtype, "float32": np.float32, "uint8": np.uint8, "float16": np.float16,
          "bfloat16": np.uint16}[dtype]
    return np.empty(n if n is not None else np.shape(x), dtype=nd)


def contiguous(x):
    if is_torch(x):
        return x.contiguous()
    return np.ascontiguousarray(x)
