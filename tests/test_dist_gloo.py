"""CPU (gloo, world size 2) checks of the host-side multi-rank logic of the
ZeRO-1 path: every rank derives the same whole-tensor shard plan
(ody_plan_shards), each rank's {nonfinite, sumsq} partial over its own
tensors, gathered in rank order, gives the unsharded step's skip / clip
decision, and a rank that never joins ends the others' collective with an
error instead of a hang."""
import os
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _decision_worker(rank, world, port, q):
    _init(rank, world, port)
    import torch
    from odyssey_b200 import plan_shards
    from odyssey_b200 import workloads as W
    from oracle import oracle as O
    wl = W.resnet18()
    owner = plan_shards(wl.numels, world)
    plans = [None] * world
    dist.all_gather_object(plans, owner)
    grads = wl.grads(100, 1)  # step 100 carries an injected inf
    stats = []
    for step_grads in (wl.grads(3, 1), grads):
        nonfinite, sumsq = 0.0, 0.0
        for i, g in enumerate(step_grads):
            if owner[i] != rank:
                continue
            u = O.unscale(g, 65536.0, dtype=O.BF16)
            nonfinite += O.count_nonfinite(u, dtype=O.BF16)
            sumsq += O.sumsq_f32(O.upcast(u, dtype=O.BF16))
        local = torch.tensor([nonfinite, sumsq], dtype=torch.float64)
        gathered = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, local)
        tot = torch.stack(gathered).sum(0)  # rank order, as the finalize kernel sums
        stats.append((float(tot[0]), float(tot[1])))
    q.put((rank, plans, stats))
    dist.destroy_process_group()


def test_two_rank_plan_and_decision():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_decision_worker, args=(r, 2, 29541, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, plans, stats = q.get(timeout=300)
        out[rank] = (plans, stats)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == out[1][0] and out[0][0][0] == out[0][0][1]
    assert out[0][1] == out[1][1]
    # unsharded oracle decision
    sys.path.insert(0, ROOT)
    from odyssey_b200 import workloads as W
    from oracle import oracle as O
    wl = W.resnet18()
    for (nonfinite, sumsq), step in zip(out[0][1], (3, 100)):
        specs = [{"numel": n, "grad_dtype": O.BF16, "quant": O.Q_NONE} for n in wl.numels]
        m = O.Model(specs, O.ADAMW, 1e-3, scaler_kwargs={"initial_scale": 65536.0})
        r = m.step(wl.grads(step, 1), 1)
        assert (nonfinite > 0) == bool(r.skipped)
        assert nonfinite == r.nonfinite
        if np.isfinite(r.sumsq):
            assert abs(sumsq - r.sumsq) <= 1e-12 * r.sumsq


def _timeout_worker(rank, world, port, q):
    _init(rank, world, port)
    import datetime
    import torch
    if rank == 1:
        q.put((rank, "left"))  # this rank leaves between steps, before the collective
        return
    t = torch.zeros(2, dtype=torch.float64)
    try:
        dist.all_reduce(t, async_op=True).wait(timeout=datetime.timedelta(seconds=3))
        q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error: " + type(e).__name__))


def test_missing_rank_ends_collective_with_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, 29547, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error")
