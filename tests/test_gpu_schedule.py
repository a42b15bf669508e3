"""GPU parity of the apply kernel's job schedule that the 1B headline runs:
requant jobs of NVFP4 per-tensor-scaled tensors interleaved with later
tensors' update jobs, each waiting (bounded, on the device) for its tensor's
update jobs to be done before it reads the tensor's amax.  The same model
under every requant placement, and at the headline's default 65,536-element
chunks, must match the oracle: NVFP4 codes, block scales and per-tensor
scales bit-exact, master weights and AdamW states within 2 ulp, identical
skip/clip decisions.  The reference computes the same values serially
(nvfp4.mojo:715-763 after adamw.mojo:123-172).

Also the failure path of that wait: a job list in which a tensor never
reaches its done count makes the wait run out after a short test limit;
the step reports ODY_ERR_DEVICE_BOUNDS and the next normal step on the same
context succeeds.  No GPU fault is involved: the kernel stops waiting and
returns."""
import ctypes as C

import numpy as np
import pytest

from odyssey_b200 import workloads as W

from test_gpu_fused import run_pair

pytestmark = pytest.mark.gpu

RQ = 0x80000000


def ctx_jobs(ctx):
    from odyssey_b200 import _lib as L
    f = L.lib().odyx_ctx_jobs
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]
    n, grid = C.c_int64(0), C.c_int32(0)
    L.check(f(ctx._ctx, None, 0, C.byref(n), C.byref(grid)))
    out = np.zeros(max(n.value, 1), np.uint32)
    L.check(f(ctx._ctx, out.ctypes.data, out.size, C.byref(n), C.byref(grid)))
    return out[: n.value], grid.value


def set_jobs(ctx, jobs, wait_ns=0):
    from odyssey_b200 import _lib as L
    f = L.lib().odyx_ctx_set_jobs
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_uint64]
    if jobs is None:
        L.check(f(ctx._ctx, None, 0, wait_ns), ctx._ctx)
    else:
        j = np.ascontiguousarray(jobs, np.uint32)
        L.check(f(ctx._ctx, j.ctypes.data, j.size, wait_ns), ctx._ctx)


def interleaved_requants(jobs):
    """Requant jobs that come before the last update job."""
    last_upd = max(i for i, j in enumerate(jobs) if not j & RQ)
    return sum(1 for j in jobs[:last_upd] if j & RQ)


@pytest.mark.parametrize("placement", ["auto", "interleaved", "at_end"])
def test_schedule_small_chunks(oracle, placement):
    """3 x 4096^2 NVFP4 + per-tensor scale at 2,048-element chunks: 24,576
    update jobs; the first two tensors are followed by more than two grid-
    widths of update jobs, so their requant jobs interleave."""
    wl = W.flat1b(ntensors=3, side=4096)
    ctx, model, res = run_pair(oracle, wl, 3, ctx_kwargs={"chunk_elems": 2048, "requant_placement": placement})
    jobs, grid = ctx_jobs(ctx)
    n_upd = sum(1 for j in jobs if not j & RQ)
    assert n_upd == 3 * 4096 * 4096 // 2048 and grid >= 148
    if placement == "at_end":
        assert interleaved_requants(jobs) == 0
    else:
        # the first two tensors' requant jobs all run between later update jobs
        assert interleaved_requants(jobs) >= 2 * 8192
    assert all(r["clipped"] for r, _ in res)
    ctx.close()


def test_schedule_default_chunks(oracle):
    """14 x 4096^2 at the size rule's own chunk length (65,536 elements, the
    1B headline's): 3,584 update jobs on the live grid, the 1B model's
    per-tensor job shape; three AdamW + clip steps."""
    wl = W.flat1b(ntensors=14, side=4096)
    ctx, model, res = run_pair(oracle, wl, 3)
    jobs, grid = ctx_jobs(ctx)
    n_upd = sum(1 for j in jobs if not j & RQ)
    assert n_upd == 14 * 256, "expected 65,536-element chunks"
    assert interleaved_requants(jobs) > 0
    ctx.close()


def test_requant_wait_limit_reports_device_bounds(oracle):
    """A job list without tensor 0's update jobs: tensor 0's requant jobs wait
    for a done count that never comes, give up after 20 ms and flag the step;
    ody_step reports ODY_ERR_DEVICE_BOUNDS.  Back on the planned list, the
    next step on the same context succeeds and clears the flag."""
    from odyssey_b200 import OdysseyError
    from odyssey_b200 import _lib as L
    wl = W.flat1b(ntensors=3, side=256)
    from odyssey_b200 import MixedPrecisionStep
    ctx = MixedPrecisionStep(wl.numels, **wl.step_kwargs())
    for i, m in enumerate(wl.master(0)):
        ctx.set_master(i, m)
    jobs, grid = ctx_jobs(ctx)
    nch = 256 * 256 // 2048  # chunk length of this small model (size rule: one tile)
    t0_chunks = set(range(nch))
    bad = [j for j in jobs if (j & RQ) or int(j) not in t0_chunks]
    assert len(bad) == len(jobs) - nch
    set_jobs(ctx, bad, wait_ns=20_000_000)
    for i, g in enumerate(wl.grads(0)):
        ctx.set_grad(i, g)
    with pytest.raises(OdysseyError) as ei:
        ctx.step(1)
    assert ei.value.code == L.ERR_DEVICE_BOUNDS
    assert "time limit" in str(ei.value)
    set_jobs(ctx, None)
    r = ctx.step(2)
    assert not r["skipped"]
    ctx.close()
