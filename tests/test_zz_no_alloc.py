"""ody_global_norm_clip_noalloc, the global-norm clip for callers that cannot
allocate GPU memory (fixed memory budgets, pre-laid-out graph memory,
real-time code): through the C ABI it must clip exactly like
ody_global_norm_clip, on two calls in a row (the shared scratch array keeps
the previous call's contents, so the second call checks that every call
starts clean), and bit for bit like the oracle's restatement of
clip_gradients_by_global_norm (gradient_clipping.mojo:313-368).  This file is
collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _clip(fn, tensors, max_norm):
    ptrs = (C.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
    numels = np.array([t.numel() for t in tensors], np.int64)
    norm = C.c_float(0.0)
    rc = fn(ptrs, numels.ctypes.data, len(tensors), max_norm, C.byref(norm))
    return rc, norm.value


def test_noalloc_matches_allocating_clip_twice(oracle):
    torch = pytest.importorskip("torch")
    from odyssey_b200 import _lib as L
    lib = L.lib()
    g = torch.Generator(device="cuda").manual_seed(3)
    for call, (sizes, scale, max_norm) in enumerate([((1, 7, 4097, 1 << 20), 3.0, 1.0),
                                                     ((33, 100000, 65536), 1e-4, 10.0)]):
        src = [torch.randn(n, device="cuda", generator=g) * scale for n in sizes]
        a = [t.clone() for t in src]
        b = [t.clone() for t in src]
        rc_a, norm_a = _clip(lib.ody_global_norm_clip, a, max_norm)
        rc_b, norm_b = _clip(lib.ody_global_norm_clip_noalloc, b, max_norm)
        assert rc_a == 0 and rc_b == 0, L.last_error()
        assert norm_b == pytest.approx(norm_a, rel=1e-6), call
        for x, y in zip(a, b):
            torch.testing.assert_close(y, x, rtol=2e-7, atol=0.0)
        # the oracle on the same inputs: the same float32 norm and the same bits
        ref = [t.cpu().numpy().copy() for t in src]
        norm_o = oracle.global_norm_clip(ref, max_norm)
        assert np.float32(norm_b) == np.float32(norm_o), call
        for y, r in zip(b, ref):
            np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), r.view(np.uint32))


def test_noalloc_rejects_too_many_tensors_and_host_memory():
    torch = pytest.importorskip("torch")
    from odyssey_b200 import _lib as L
    lib = L.lib()
    t = torch.ones(4, device="cuda")
    rc, _ = _clip(lib.ody_global_norm_clip_noalloc, [t] * 1025, 1.0)
    assert rc == L.ERR_SHAPE and "at most 1024" in L.last_error()
    h = np.ones(4, np.float32)
    ptrs = (C.c_void_p * 1)(h.ctypes.data)
    n = np.array([4], np.int64)
    norm = C.c_float(0)
    assert lib.ody_global_norm_clip_noalloc(ptrs, n.ctypes.data, 1, 1.0, C.byref(norm)) == L.ERR_ARG
    assert "not device memory" in L.last_error()


def test_noalloc_refuses_another_gpus_memory():
    """Gradients on a GPU other than the calling thread's current one are
    refused before any launch (without peer access the kernels would fault)."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from odyssey_b200 import _lib as L
    lib = L.lib()
    t = torch.ones(4, device="cuda:1")
    torch.cuda.set_device(0)
    rc, _ = _clip(lib.ody_global_norm_clip_noalloc, [t], 1.0)
    assert rc == L.ERR_ARG and "not of the current GPU" in L.last_error()
    assert torch.equal(t.cpu(), torch.ones(4))
