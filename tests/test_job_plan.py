"""The apply kernel's job list (host logic, no GPU): every update chunk once,
every requant chunk of a per-tensor-scaled tensor once and only after all of
its tensor's update jobs, tensors largest first (stable), requant jobs of a
large model interleaved two grid-widths after their tensor, those of a small
model all at the end.  Reached through the odyx_plan_jobs test hook."""
import ctypes as C

import numpy as np
import pytest

RQ = 0x80000000
NVT, FP8T, NONE, MX = 8, 5, 0, 6


@pytest.fixture(scope="module")
def lib():
    from odyssey_b200 import _lib as L
    from odyssey_b200.build import build
    build()
    f = L.lib().odyx_plan_jobs
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p]
    return f


def plan(lib, nchunks, quant, W):
    nc = np.array(nchunks, np.int32)
    q = np.array(quant, np.int32)
    n = C.c_int64(0)
    assert lib(nc.ctypes.data, q.ctypes.data, len(nc), W, None, 0, C.byref(n)) == 0
    out = np.zeros(max(n.value, 1), np.uint32)
    assert lib(nc.ctypes.data, q.ctypes.data, len(nc), W, out.ctypes.data, out.size, C.byref(n)) == 0
    return out[: n.value]


def check(jobs, nchunks, quant, W):
    first = np.concatenate([[0], np.cumsum(nchunks)[:-1]]).astype(int)
    owner = np.repeat(np.arange(len(nchunks)), nchunks)
    upd = [int(j) for j in jobs if not j & RQ]
    rq = [int(j) & ~RQ for j in jobs if j & RQ]
    assert sorted(upd) == list(range(sum(nchunks)))
    want_rq = [c for t in range(len(nchunks)) if quant[t] in (NVT, FP8T) for c in range(first[t], first[t] + nchunks[t])]
    assert sorted(rq) == sorted(want_rq)
    pos = {(bool(j & RQ), int(j) & ~RQ): i for i, j in enumerate(jobs)}
    for c in rq:
        t = owner[c]
        last_upd = max(pos[(False, k)] for k in range(first[t], first[t] + nchunks[t]))
        assert pos[(True, c)] > last_upd
    # tensors' update jobs in descending size, stable
    order = []
    for j in upd:
        t = owner[j]
        if not order or order[-1] != t:
            order.append(t)
    assert order == sorted(range(len(nchunks)), key=lambda t: -nchunks[t])
    return pos, owner, first


def test_large_model_interleaves(lib):
    nchunks, quant, W = [256] * 16, [NVT] * 16, 148
    jobs = plan(lib, nchunks, quant, W)
    pos, owner, first = check(jobs, nchunks, quant, W)
    # tensor 0's requant jobs start two grid-widths after its last update job
    last_upd0 = max(pos[(False, k)] for k in range(0, 256))
    first_rq0 = min(pos[(True, k)] for k in range(0, 256))
    assert 2 * W <= first_rq0 - last_upd0 <= 2 * W + 4
    # and are interleaved with later update jobs (at most two per update job)
    run = 0
    for j in jobs[first_rq0: first_rq0 + 200]:
        run = run + 1 if j & RQ else 0
        assert run <= 2


def test_small_model_requant_at_end(lib):
    nchunks = [3, 40, 7, 40, 1]
    quant = [FP8T, NONE, NVT, MX, FP8T]
    jobs = plan(lib, nchunks, quant, 148)
    check(jobs, nchunks, quant, 148)
    n_upd = sum(nchunks)
    assert all(not (j & RQ) for j in jobs[:n_upd]) and all(j & RQ for j in jobs[n_upd:])


@pytest.mark.parametrize("seed", range(20))
def test_random_models(lib, seed):
    rng = np.random.default_rng(seed)
    nt = int(rng.integers(1, 40))
    nchunks = [int(x) for x in rng.integers(1, 300, nt)]
    quant = [int(x) for x in rng.choice([NONE, MX, NVT, FP8T, 1], nt)]
    W = int(rng.choice([1, 7, 148, 592]))
    check(plan(lib, nchunks, quant, W), nchunks, quant, W)


def test_small_buffer_refused(lib):
    nc = np.array([4], np.int32)
    q = np.array([NVT], np.int32)
    out = np.zeros(3, np.uint32)
    n = C.c_int64(0)
    assert lib(nc.ctypes.data, q.ctypes.data, 1, 4, out.ctypes.data, 3, C.byref(n)) != 0
