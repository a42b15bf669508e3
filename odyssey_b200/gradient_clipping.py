"""Mirror of src/odyssey/training/gradient_clipping.mojo:273-368 over libodyssey_mp.so."""
import ctypes as C

import numpy as np

from . import _lib as L


def clip_gradients_by_global_norm(gradients, max_norm):
    """Clip a list of float32 gradient tensors in place; returns the pre-clip
    global norm (gradient_clipping.mojo:313-368)."""
    if max_norm <= 0.0:
        raise L.OdysseyError("max_norm must be positive, got: " + str(max_norm), L.ERR_ARG)
    for g in gradients:
        if L.dtype_code(g) != L.F32:
            raise L.OdysseyError("clip_gradients_by_global_norm takes float32 gradients", L.ERR_DTYPE)
        if (L.is_torch(g) and not g.is_contiguous()) or (not L.is_torch(g) and not g.flags["C_CONTIGUOUS"]):
            raise L.OdysseyError("gradients must be contiguous (clipped in place)", L.ERR_ARG)
    n = len(gradients)
    ptrs = (C.c_void_p * max(n, 1))(*[L.ptr(g) for g in gradients])
    numels = np.array([L.numel(g) for g in gradients] or [0], np.int64)
    norm = C.c_float(0.0)
    L.check(L.lib().ody_global_norm_clip(ptrs, numels.ctypes.data, n, max_norm, C.byref(norm)))
    return norm.value


def compute_gradient_norm_list(gradients):
    """Global L2 norm of a list of float32 gradients (gradient_clipping.mojo:273-310)."""
    copies = [np.array(g, dtype=np.float32, copy=True) if not L.is_torch(g) else g.float().contiguous().clone()
              for g in gradients]
    return clip_gradients_by_global_norm(copies, float(np.finfo(np.float32).max))


def _clip_variant(tensors, max_norm, mode, name):
    for g in tensors:
        if L.dtype_code(g) != L.F32:
            raise L.OdysseyError(f"{name} takes float32 tensors", L.ERR_DTYPE)
        if (L.is_torch(g) and not g.is_contiguous()) or (not L.is_torch(g) and not g.flags["C_CONTIGUOUS"]):
            raise L.OdysseyError("tensors must be contiguous (clipped in place)", L.ERR_ARG)
    n = len(tensors)
    ptrs = (C.c_void_p * max(n, 1))(*[L.ptr(g) for g in tensors])
    numels = np.array([L.numel(g) for g in tensors] or [0], np.int64)
    norm = C.c_double(0.0)
    L.check(L.lib().ody_clip_global_norm_variant(ptrs, numels.ctypes.data, n, float(max_norm), mode,
                                                 C.byref(norm)))
    return norm.value


def clip_grad_global_norm_(grads, max_norm):
    """core/numerical_safety.mojo:760-815: float32 squares, factor
    max_norm / norm (no +1e-6) applied as a float32 multiplier when
    norm > max_norm and norm > 0; returns the float64 norm before clipping."""
    return _clip_variant(grads, max_norm, 0, "clip_grad_global_norm_")


def clip_global_norm(tensors, max_norm):
    """training/optimizers/optimizer_utils.mojo:303-348: float64 squares,
    each value scaled in float64 and rounded to float32; returns the float64
    norm before clipping."""
    return _clip_variant(tensors, max_norm, 1, "clip_global_norm")
