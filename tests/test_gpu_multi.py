"""Multi-GPU parity: the ZeRO-1-sharded step on 2 GPUs (one process each,
NCCL allgather of the per-rank {nonfinite, sumsq}) against the oracle's
unsharded step.  Every rank must take the identical skip/backoff decision,
and each rank's tensors must match the oracle (master within 2 ulp, codes
bit-exact).  Skipped when fewer than 2 GPUs are visible."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


GDT = {"float32": 0, "float16": 1, "bfloat16": 2}
OPT = {"sgd": 0, "adam": 1, "adamw": 2}
QK = {"none": 0, "fp16": 1, "bf16": 2, "fp8": 3, "bf8": 4, "fp8_tensor": 5, "mxfp4": 6, "nvfp4": 7,
      "nvfp4_tensor": 8}


def dp_reduce(wl, step, world):
    """The data-parallel gradient: the ranks' gradients upcast to float32,
    summed in rank order (one rounding per add), rounded to the gradient
    dtype."""
    per = [wl.grads(step, 1 + r) for r in range(world)]
    out = []
    for i in range(len(wl.numels)):
        acc = None
        for r in range(world):
            g = per[r][i]
            x = W_bf16_to_f32(g) if wl.grad_dtype == "bfloat16" else g.astype(np.float32)
            acc = x.copy() if acc is None else (acc + x).astype(np.float32)
        if wl.grad_dtype == "bfloat16":
            out.append(W_f32_to_bf16(acc))
        elif wl.grad_dtype == "float16":
            out.append(acc.astype(np.float16))
        else:
            out.append(acc)
    return out


def W_bf16_to_f32(h):
    from odyssey_b200 import workloads as W
    return W.bf16_bits_to_f32(h)


def W_f32_to_bf16(x):
    """float32 -> bfloat16 bits, round to nearest even, NaN kept NaN."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = ((u[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return r


@pytest.mark.parametrize("which,port", [("resnet18", 29533), ("flat", 29534), ("dp_resnet18", 29535),
                                        ("dp_flat", 29536)])
def test_two_rank_matches_unsharded_oracle(oracle, tmp_path, which, port):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    steps, inf_every = 5, 3
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "dist_worker.py"), str(tmp_path), str(steps), str(inf_every), which]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    # identical decisions on both ranks
    np.testing.assert_array_equal(ranks[0]["results"], ranks[1]["results"])

    from odyssey_b200 import workloads as W
    dp = which.startswith("dp_")
    base = which[3:] if dp else which
    wl = W.resnet18() if base == "resnet18" else W.flat1b(ntensors=4, side=512)
    wl.inf_every = inf_every
    kw = wl.step_kwargs()
    hy = wl.hyper
    specs = [{"numel": n, "grad_dtype": GDT[wl.grad_dtype], "quant": QK[wl.quant]} for n in wl.numels]
    sk = {k: kw[k] for k in ("initial_scale", "growth_factor", "backoff_factor", "growth_interval", "min_scale",
                             "max_scale") if k in kw}
    model = oracle.Model(specs, OPT[wl.optimizer], hy["learning_rate"], beta1=hy.get("beta1", 0.9),
                         beta2=hy.get("beta2", 0.999), epsilon=hy.get("epsilon", 1e-8),
                         weight_decay=hy.get("weight_decay", 0.0), clip_enabled=wl.clip is not None,
                         max_norm=wl.clip or 1.0, scaler_kwargs=sk)
    for i, m in enumerate(wl.master(0)):
        model.master[i][:] = m
    t = 1
    for s in range(steps):
        r = model.step(dp_reduce(wl, s, 2) if dp else wl.grads(s, 1), t)
        got = ranks[0]["results"][s]
        assert got[0] == r.skipped and got[1] == r.nonfinite and got[4] == r.scale_next
        if np.isfinite(r.sumsq):
            assert abs(got[2] - r.sumsq) <= 1e-12 * r.sumsq
        if not r.skipped:
            t += 1
    seen = []
    for z in ranks:
        for i in z["owned"]:
            seen.append(int(i))
            d = np.abs(z[f"master{i}"].view(np.int32).astype(np.int64) - model.master[i].view(np.int32))
            assert d.max() <= 2, i
            np.testing.assert_array_equal(z[f"codes{i}"], model.qout[i][: z[f"codes{i}"].size])
            assert z[f"scale{i}"] == model.qscale[i][0]
    assert sorted(seen) == list(range(len(wl.numels)))
    # the gathered model on each rank: every tensor's codes and scale
    for z in ranks:
        for i in range(len(wl.numels)):
            np.testing.assert_array_equal(z[f"gathered{i}"], model.qout[i][: z[f"gathered{i}"].size])
            assert z["scales"][i] == model.qscale[i][0]
