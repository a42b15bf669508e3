"""Mirror of AnyTensor.to_/from_{fp8,bf8,mxfp4,nvfp4}
(src/odyssey/tensor/any_tensor.mojo:1946-2427, tensor_dtype_conv.mojo:13-494)
over libodyssey_mp.so.

A quantised tensor is a flat uint8 buffer in the reference's layout (FP8:
one byte per element; MXFP4: 17-byte blocks of 16 code bytes + 1 E8M0
byte; NVFP4: 9-byte blocks of 8 code bytes + 1 E4M3 byte; element 2i in
the high nibble) plus the original element count
(AnyTensor._original_numel_quantized, any_tensor.mojo:140) and, for the
per-tensor-scaled kinds, the float32 tensor scale.
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L


@dataclass
class QuantizedTensor:
    data: object          # uint8 buffer (numpy array or torch tensor)
    kind: int
    original_numel: int
    tensor_scale: float = 1.0


def quantize(x, kind, dtype=None):
    """x: float32 or bfloat16 (torch bfloat16, or numpy uint16 with dtype='bfloat16')."""
    code = L.dtype_code(x, dtype)
    if code == L.F16:
        # the reference accepts float16 sources by an exact upcast
        from .mixed_precision import convert_to_fp32_master
        x, code = convert_to_fp32_master(x), L.F32
    n = L.numel(x)
    if n == 0:
        raise L.OdysseyError("cannot quantize an empty tensor", L.ERR_SHAPE)
    src = L.contiguous(x)
    out = L.empty_like(src, "uint8", L.quant_bytes(kind, n))
    ts = C.c_float(1.0)
    L.check(L.lib().ody_quantize(kind, L.ptr(src), code, n, L.ptr(out), C.byref(ts)))
    return QuantizedTensor(out, kind, n, ts.value)


def dequantize(q):
    """QuantizedTensor -> float32 values (1-D, original_numel long)."""
    need = L.quant_bytes(q.kind, q.original_numel)
    if L.numel(q.data) != need:
        raise L.OdysseyError(f"quantised buffer has {L.numel(q.data)} bytes, expected {need}", L.ERR_SHAPE)
    data = L.contiguous(q.data)
    out = L.empty_like(data, "float32", q.original_numel)
    L.check(L.lib().ody_dequantize(q.kind, L.ptr(data), q.original_numel, q.tensor_scale, L.ptr(out)))
    return out


def _reference_source(x, dtype, method):
    """The source checks of AnyTensor.to_fp8/to_bf8/to_mxfp4/to_nvfp4
    (tensor_dtype_conv.mojo:21-36 and 259-279): bfloat16 is rejected,
    float16/float32/float64 are accepted (float64 rounded to float32 as the
    reference's .cast[DType.float32] does), anything else is rejected."""
    bf16 = dtype in ("bfloat16", L.BF16)
    name = None
    if L.is_torch(x):
        name = str(x.dtype).replace("torch.", "")
        bf16 = bf16 or name == "bfloat16"
    else:
        name = np.asarray(x).dtype.name
    if bf16:
        raise L.OdysseyError(f"{method} does not support bfloat16: the bfloat16 conversion path does not correctly "
                             "round-trip through the Float32 intermediate representation", L.ERR_DTYPE)
    if dtype is None and name == "float64":
        return x.float() if L.is_torch(x) else np.asarray(x, np.float32)
    if dtype is None and name not in ("float16", "float32"):
        raise L.OdysseyError(f"{method} requires a floating-point tensor", L.ERR_DTYPE)
    return x


def to_fp8(x, dtype=None):
    """AnyTensor.to_fp8 (any_tensor.mojo:1946-2002): float16/32/64 sources."""
    return quantize(_reference_source(x, dtype, "to_fp8()"), L.Q_FP8_E4M3, dtype)


def to_bf8(x, dtype=None):
    """AnyTensor.to_bf8 (any_tensor.mojo:2165-2220): float16/32/64 sources."""
    return quantize(_reference_source(x, dtype, "to_bf8()"), L.Q_FP8_E5M2, dtype)


def to_fp8_tensor_scaled(x, dtype=None):
    """Extension: FP8 E4M3 with a per-tensor scale; bfloat16 sources are
    accepted (upcast exactly)."""
    return quantize(x, L.Q_FP8_E4M3_TENSOR, dtype)


def to_mxfp4(x, dtype=None):
    """AnyTensor.to_mxfp4 (any_tensor.mojo:2237-2302): float16/32/64 sources."""
    return quantize(_reference_source(x, dtype, "to_mxfp4()"), L.Q_MXFP4, dtype)


def to_mxfp4_ocp(x, dtype=None):
    """MXFP4 by the OCP Microscaling Formats v1.0 rule (extension, no
    reference counterpart): E8M0 = floor(log2 amax) - 2 per 32-element
    block, elements rounded to nearest even on the E2M1 grid.  float32 or
    bfloat16 sources; decode with dequantize(q, ...) or from_mxfp4_ocp."""
    return quantize(x, L.Q_MXFP4_OCP, dtype)


def to_nvfp4(x, dtype=None):
    """AnyTensor.to_nvfp4 (any_tensor.mojo:2329-2401): float16/32/64 sources;
    bfloat16 through quantize() or to_nvfp4_tensor_scaled (extensions)."""
    return quantize(_reference_source(x, dtype, "to_nvfp4()"), L.Q_NVFP4, dtype)


def to_nvfp4_tensor_scaled(x, dtype=None):
    """Extension: NVFP4 with a per-tensor scale; bfloat16 sources are
    accepted (upcast exactly)."""
    return quantize(x, L.Q_NVFP4_TENSOR, dtype)


def _from(q, kind, block, what):
    if isinstance(q, QuantizedTensor):
        return dequantize(q)
    # tensor_dtype_conv.mojo:78-79, 227-228, 380-385, 444-449
    is_u8 = str(q.dtype) == "torch.uint8" if L.is_torch(q) else np.asarray(q).dtype == np.uint8
    if not is_u8:
        raise L.OdysseyError(f"from_{what.lower()}() requires a uint8 tensor ({what}-encoded)", L.ERR_DTYPE)
    nbytes = L.numel(q)
    if block and nbytes % block:
        raise L.OdysseyError(f"{what} tensor size must be multiple of {block} bytes", L.ERR_SHAPE)
    n = nbytes // block * (32 if block == 17 else 16) if block else nbytes
    return dequantize(QuantizedTensor(q, kind, n))


def from_fp8(q):
    return _from(q, L.Q_FP8_E4M3, 0, "FP8")


def from_bf8(q):
    return _from(q, L.Q_FP8_E5M2, 0, "BF8")


def from_mxfp4(q):
    """tensor_dtype_conv.mojo:369-430 (padded length when the original numel is unknown)."""
    return _from(q, L.Q_MXFP4, 17, "MXFP4")


def from_nvfp4(q):
    """tensor_dtype_conv.mojo:433-494."""
    return _from(q, L.Q_NVFP4, 9, "NVFP4")


class _FP4Single:
    """FP4 singles: one E2M1 code per value, each with its own power-of-two
    scale byte (MXFP4 / NVFP4 scalar types, src/odyssey/core/types/
    mxfp4.mojo:279-491 and nvfp4.mojo:265-481), over arrays of values."""

    kind = None

    @classmethod
    def _encode(cls, x, seeds):
        src = L.contiguous(x)
        n = L.numel(src)
        if n == 0:
            raise L.OdysseyError("cannot convert an empty tensor", L.ERR_SHAPE)
        if L.dtype_code(src) != L.F32:
            raise L.OdysseyError("FP4 singles convert float32 values", L.ERR_DTYPE)
        sd = None
        if seeds is not None:
            sd = np.ascontiguousarray(seeds, np.uint64) if not L.is_torch(seeds) else seeds.contiguous()
            if L.numel(sd) != n:
                raise L.OdysseyError("one seed per value", L.ERR_SHAPE)
        vals, scs = L.empty_like(src, "uint8", n), L.empty_like(src, "uint8", n)
        L.check(L.lib().ody_fp4_single_encode(cls.kind, L.ptr(src), n, L.ptr(sd), L.ptr(vals), L.ptr(scs)))
        return vals, scs

    @classmethod
    def from_float32(cls, x):
        """from_float32 per value -> (codes, scale bytes)."""
        return cls._encode(x, None)

    @classmethod
    def from_float32_stochastic(cls, x, seeds):
        """from_float32_stochastic per value with its seed -> (codes, scale bytes)."""
        return cls._encode(x, seeds)

    @classmethod
    def to_float32(cls, values, scales):
        v, s = L.contiguous(values), L.contiguous(scales)
        n = L.numel(v)
        if n == 0 or L.numel(s) != n:
            raise L.OdysseyError("values and scales must be non-empty and of one length", L.ERR_SHAPE)
        out = L.empty_like(v, "float32", n)
        L.check(L.lib().ody_fp4_single_decode(cls.kind, L.ptr(v), L.ptr(s), n, L.ptr(out)))
        return out


class MXFP4(_FP4Single):
    """MXFP4 singles (E8M0 scale bytes)."""
    kind = L.QUANT_NAMES["mxfp4"]


class NVFP4(_FP4Single):
    """NVFP4 singles (E4M3 scale bytes)."""
    kind = L.QUANT_NAMES["nvfp4"]
