"""The apply kernel's job list (host logic, no GPU): every update chunk once,
every requant chunk of a per-tensor-scaled tensor once and only after all of
its tensor's update jobs, tensors largest first (stable).  Interleaved
placement puts a tensor's requant jobs two grid-widths after its last update
job when enough update jobs follow it (decided per tensor); at-end placement
puts them all last; auto is interleaved.  Reached through the odyx_plan_jobs test hook."""
import ctypes as C

import numpy as np
import pytest

RQ = 0x80000000
NVT, FP8T, NONE, MX = 8, 5, 0, 6
AUTO, INTER, END = 0, 1, 2


@pytest.fixture(scope="module")
def lib():
    from odyssey_b200 import _lib as L
    from odyssey_b200.build import build
    build()
    f = L.lib().odyx_plan_jobs
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p]
    return f


def plan(lib, nchunks, quant, W, placement=AUTO):
    nc = np.array(nchunks, np.int32)
    q = np.array(quant, np.int32)
    n = C.c_int64(0)
    assert lib(nc.ctypes.data, q.ctypes.data, len(nc), W, placement, None, 0, C.byref(n)) == 0
    out = np.zeros(max(n.value, 1), np.uint32)
    assert lib(nc.ctypes.data, q.ctypes.data, len(nc), W, placement, out.ctypes.data, out.size, C.byref(n)) == 0
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
    """Fewer than two grid-widths of update jobs after every tensor: all
    requant jobs come last even under the interleaved placement."""
    nchunks = [3, 40, 7, 40, 1]
    quant = [FP8T, NONE, NVT, MX, FP8T]
    jobs = plan(lib, nchunks, quant, 148)
    check(jobs, nchunks, quant, 148)
    n_upd = sum(nchunks)
    assert all(not (j & RQ) for j in jobs[:n_upd]) and all(j & RQ for j in jobs[n_upd:])


def interleaved_tensors(jobs, nchunks, quant):
    """Tensors whose first requant job comes before the last update job."""
    last_upd = max(i for i, j in enumerate(jobs) if not j & RQ)
    owner = np.repeat(np.arange(len(nchunks)), nchunks)
    return sorted({int(owner[int(j) & ~RQ]) for i, j in enumerate(jobs) if j & RQ and i < last_upd})


def test_few_large_tensors_interleave_per_tensor(lib):
    """The 1B model on 8 ranks: 8 tensors of 512 chunks per rank, a 592-CTA
    grid (4,096 update jobs, under eight grid-widths).  Every tensor with two
    grid-widths (1,184) of update jobs after it interleaves; the last three
    (1,024 or fewer update jobs after them) cannot."""
    nchunks, quant, W = [512] * 8, [NVT] * 8, 592
    for placement in (AUTO, INTER):
        jobs = plan(lib, nchunks, quant, W, placement)
        check(jobs, nchunks, quant, W)
        assert interleaved_tensors(jobs, nchunks, quant) == [0, 1, 2, 3, 4]
    jobs = plan(lib, nchunks, quant, W, END)
    check(jobs, nchunks, quant, W)
    assert interleaved_tensors(jobs, nchunks, quant) == []


def test_auto_is_interleaved(lib):
    """Auto placement is the interleaved one for every model size, ResNet-18-
    like mixes of tensor sizes included."""
    W = 592
    rn = [576] * 2 + [288] * 3 + [144] * 4 + [72] * 8 + [16] * 10
    q = [FP8T] * len(rn)
    for nchunks, quant in (([256] * 16, [NVT] * 16), (rn, q), ([3, 40, 7, 40, 1], [FP8T, NONE, NVT, MX, FP8T])):
        a, b = plan(lib, nchunks, quant, W), plan(lib, nchunks, quant, W, INTER)
        np.testing.assert_array_equal(a, b)
    assert interleaved_tensors(plan(lib, rn, q, W), rn, q)


@pytest.mark.parametrize("seed", range(20))
def test_random_models(lib, seed):
    rng = np.random.default_rng(seed)
    nt = int(rng.integers(1, 40))
    nchunks = [int(x) for x in rng.integers(1, 300, nt)]
    quant = [int(x) for x in rng.choice([NONE, MX, NVT, FP8T, 1], nt)]
    W = int(rng.choice([1, 7, 148, 592]))
    for placement in (AUTO, INTER, END):
        check(plan(lib, nchunks, quant, W, placement), nchunks, quant, W)


def test_small_buffer_refused(lib):
    nc = np.array([4], np.int32)
    q = np.array([NVT], np.int32)
    out = np.zeros(3, np.uint32)
    n = C.c_int64(0)
    assert lib(nc.ctypes.data, q.ctypes.data, 1, 4, AUTO, out.ctypes.data, 3, C.byref(n)) != 0
