"""Rank program of the multi-GPU parity test (tests/test_gpu_multi.py).

Launched by torch.distributed.run, one process per GPU, on the ResNet-18
workload (unequal shards) or a 4-tensor flat model (equal shards: the
gather takes its allgather path); with a "dp_" prefix every rank feeds its
own full-model gradients and the step reduce-scatters them.  Every rank generates the same seeded
model and gradients, builds a ZeRO-1-sharded
MixedPrecisionStep (whole tensors per rank, NCCL allgather of the
{nonfinite, sumsq} pair), runs the steps, and saves its owned tensors'
master weights and codes plus the step results to <out>/rank<r>.npz.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    out, steps, inf_every = sys.argv[1], int(sys.argv[2]), int(sys.argv[3])
    which = sys.argv[4] if len(sys.argv) > 4 else "resnet18"
    import torch
    import torch.distributed as dist

    from odyssey_b200 import MixedPrecisionStep
    from odyssey_b200 import workloads as W

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    rank = dist.get_rank()
    dp = which.startswith("dp_")
    base = which[3:] if dp else which
    wl = W.resnet18() if base == "resnet18" else W.flat1b(ntensors=4, side=512)
    wl.inf_every = inf_every
    kw = wl.step_kwargs()
    kw["device"] = local
    ctx = MixedPrecisionStep.from_process_group(wl.numels, **kw)
    if dp:
        ctx.dp_attach()
    master = wl.master(0)
    for i in ctx.owned:
        ctx.set_master(i, master[i])
    res = []
    t = 1
    for s in range(steps):
        if dp:
            # data-parallel: every rank's own full-model gradients
            for i, g in enumerate(wl.grads(s, 1 + rank)):
                ctx.set_dp_grad(i, g)
        else:
            grads = wl.grads(s, 1)
            for i in ctx.owned:
                ctx.set_grad(i, grads[i])
        r = ctx.step(t)
        res.append([r["skipped"], r["nonfinite_count"], r["sumsq"], r["grad_norm"], r["scale_next"]])
        if not r["skipped"]:
            t += 1
    buf, scales = ctx.gather_quant()
    gathered = buf.cpu().numpy()
    arrays = {"owned": np.array(ctx.owned), "results": np.array(res, np.float64), "scales": scales.cpu().numpy()}
    for i in range(len(wl.numels)):
        off, nb, _ = ctx.quant_layout(i)
        arrays[f"gathered{i}"] = gathered[off:off + nb]
    for i in ctx.owned:
        arrays[f"master{i}"] = ctx.master(i)
        q = ctx.get_quant(i)
        arrays[f"codes{i}"] = q.data
        arrays[f"scale{i}"] = np.float32(q.tensor_scale)
    np.savez(os.path.join(out, f"rank{rank}.npz"), **arrays)
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
