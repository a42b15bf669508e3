"""Benchmark of the fused mixed-precision step (BASELINE.json metric:
"fused mixed-precision step: params/s & HBM GB/s (% of peak), 1/2/4/8 B200").

Workload (configs[4], the 1B-param flat model the target is quoted on; it
fits one B200): 64 x 4096x4096 float32 master weights ~ N(0, 0.02^2),
bfloat16 gradients ~ N(0, 1e-3^2) x loss scale 4096, AdamW (lr 1e-3, betas
0.9/0.999, eps 1e-8, wd 0.01) + global-norm clip 1.0, NVFP4 requant with a
per-tensor scale.  With N GPUs the 64 tensors are ZeRO-1-sharded (8 whole
tensors per rank at N=8): total work is fixed, scaling is "strong".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the hot path (stats -> [allgather] -> update ->
requant) over the whole model.  `value` is params/s of the whole job with
inputs resident in HBM; `e2e` is the same metric through the public C ABI
with the gradients copied from pinned host memory every step and the step
result read back.  The reference arm times the CPU restatement of the
reference (oracle/) on the host cores over a bounded sample.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused mixed-precision step: params/s & HBM GB/s (% of peak), 1/2/4/8 B200"
NT, SIDE = 64, 4096
PER = SIDE * SIDE
TOTAL = NT * PER
ALG_BYTES_STEP = 26.5625        # grads 2 + master/m/v r+w 24 + NVFP4 codes 0.5625 (B/param)
ALG_BYTES_UPDATE = 26.5625      # apply kernel: grads 2 + master/m/v r+w 24 + NVFP4 codes 0.5625
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes per param of one apply_kernel launch, measured with ncu
# (dram__bytes_read.sum + dram__bytes_write.sum of the 8-tensor case
# `--tensors 8`, divided by its 134,217,728 params; traffic grows with the
# params a launch processes)
TRAFFIC_BYTES_PER_PARAM_APPLY = 30.45


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        try:
            d = json.load(open(p))
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu):
        self.gpu, self.p, self.out = gpu, None, None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.out = ""

    def summary(self):
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_info():
    model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return model, os.cpu_count()


def cpu_reference_sample(seconds=12.0, ntensors=1):
    """The oracle (CPU restatement of the reference path) on the host cores:
    the same AdamW + clip + NVFP4-per-tensor step over `ntensors` of the
    workload's 4096x4096 tensors, repeated for about `seconds`."""
    from oracle import oracle as O
    from odyssey_b200 import workloads as W
    O.build()
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    wl = W.flat1b(ntensors=ntensors, side=SIDE)
    specs = [{"numel": n, "grad_dtype": O.BF16, "quant": O.Q_NVFP4_TENSOR} for n in wl.numels]
    m = O.Model(specs, O.ADAMW, 1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01,
                clip_enabled=True, max_norm=1.0, scaler_kwargs={"initial_scale": 4096.0})
    for i, x in enumerate(wl.master(0)):
        m.master[i][:] = x
    grads = wl.grads(0)
    m.step(grads, 1)  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    t = 2
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        m.step(grads, t)
        times.append(time.perf_counter() - t0)
        t += 1
    sec = statistics.median(times)
    params = sum(wl.numels)
    return {"value": params / sec, "unit": "params/s", "cores": threads, "kind": "port",
            "sample": f"{ntensors} x 4096x4096 tensor(s) ({params} params) of the 1B workload, "
                      f"AdamW+clip+NVFP4-per-tensor, {len(times)} steps, median {sec * 1e3:.1f} ms/step, "
                      f"{threads} OpenMP threads on {cpu_info()[0]}"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cb = cpu_reference_sample(seconds=max(3.0, min(30.0, 2.0 * args.steps)))
    line = {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "params/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": TOTAL / cb["value"] * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_dict(world),
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "params/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def config_dict(world):
    name = "flat1b_adamw_clip_bf16_nvfp4 (configs[4])" if NT == 64 else f"flat_{NT}x4096^2 (profiling case)"
    return {"workload": name, "params": TOTAL, "tensors": NT,
            "tensor_shape": [SIDE, SIDE], "grad_dtype": "bf16", "master_dtype": "f32", "optimizer": "adamw",
            "clip_max_norm": 1.0, "quant": "nvfp4 + per-tensor f32 scale", "loss_scale": 4096.0,
            "parallelism": f"zero1 whole-tensor shards x{world}",
            "l2": "inputs larger than L2 (>= 3.5 GB/step/GPU), no flush needed"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tensors", type=int, default=64,
                    help="number of 4096x4096 tensors (64 = the 1B workload; fewer only for profiling)")
    ap.add_argument("--quant", default="nvfp4_tensor",
                    help="re-quantisation kind (the workload's is nvfp4_tensor; others only for comparisons)")
    args = ap.parse_args()
    global NT, TOTAL
    NT, TOTAL = args.tensors, args.tensors * PER
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    import odyssey_b200 as ody
    from odyssey_b200 import _lib as L
    from odyssey_b200.workloads import flat1b

    torch.cuda.set_device(local)
    if world > 1:
        # host-side plumbing only (NCCL id broadcast, barriers, max over ranks);
        # the step's own exchange runs on the library's NCCL communicator
        dist.init_process_group("gloo")
    wl = flat1b(ntensors=NT)
    kw = wl.step_kwargs()
    kw["device"] = local
    kw["quant"] = args.quant
    if world > 1:
        ctx = ody.MixedPrecisionStep.from_process_group(wl.numels, **kw)
    else:
        ctx = ody.MixedPrecisionStep(wl.numels, **kw)
    owned = ctx.owned
    nloc = len(owned) * PER

    # synthetic inputs generated on the device (seeded), copied into the arenas
    gen = torch.Generator(device="cuda")
    for i in owned:
        gen.manual_seed(1000 + i)
        m = torch.randn(PER, device="cuda", generator=gen) * 0.02
        ctx.upload(L.BUF_MASTER, i, m)
        gen.manual_seed(5000 + i)
        g = (torch.randn(PER, device="cuda", generator=gen) * (1e-3 * 4096.0)).to(torch.bfloat16)
        ctx.upload(L.BUF_GRAD, i, g)
        del m, g
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    t = 1
    w0 = time.perf_counter()
    for _ in range(args.warmup):
        ctx.step(t)
        t += 1
    # every rank must run the same number of steps (each step has a
    # collective): the untimed clock-warm-up count is agreed from the slowest
    # rank's warm-up time
    per_step = torch.tensor([(time.perf_counter() - w0) / max(args.warmup, 1)], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(per_step, op=dist.ReduceOp.MAX)
    n_clock_warm = max(3, min(5000, int(1.5 / max(per_step.item(), 1e-6))))
    stream = torch.cuda.ExternalStream(ctx.stream_handle())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.set_timing(True)
    ctx.pass_times()
    barrier()
    with Clocks(local) as clk:
        # keep the GPU loaded while the clock sampler starts (untimed steps)
        for _ in range(n_clock_warm):
            ctx.step(t)
            t += 1
        ctx.pass_times()
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            ctx.step_async(t)
            t += 1
        ev1.record(stream)
        res = ctx.wait()
        ev1.synchronize()
    barrier()
    ms_total = ev0.elapsed_time(ev1)
    passes, nsteps = ctx.pass_times()
    ctx.set_timing(False)
    if world > 1:
        x = torch.tensor([ms_total, passes["update"], passes["stats"], passes["requant"], passes["exchange"]],
                         dtype=torch.float64)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        ms_total, passes["update"], passes["stats"], passes["requant"], passes["exchange"] = x.tolist()
    ms_step = ms_total / args.steps
    value = TOTAL / (ms_step * 1e-3)

    # ---- end to end through the C ABI: pinned host gradients -> step -> result
    pinned = [torch.empty(PER, dtype=torch.bfloat16, pin_memory=True) for _ in owned]
    for k, i in enumerate(owned):
        pinned[k].copy_(torch.from_numpy(ctx.download(L.BUF_GRAD, i)).view(torch.bfloat16))
    lib = L.lib()
    for _ in range(1):
        for k, i in enumerate(owned):
            L.check(lib.ody_upload_async(ctx._ctx, L.BUF_GRAD, i, pinned[k].data_ptr(), PER * 2), ctx._ctx)
        ctx.step(t)
        t += 1
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.e2e_steps):
        for k, i in enumerate(owned):
            L.check(lib.ody_upload_async(ctx._ctx, L.BUF_GRAD, i, pinned[k].data_ptr(), PER * 2), ctx._ctx)
        ctx.step(t)  # synchronous: includes the device->host read of the step result
        t += 1
    e1.record(stream)
    e1.synchronize()
    wall = time.perf_counter() - w0
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        x = torch.tensor([e2e_ms], dtype=torch.float64)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        e2e_ms = x.item()

    if rank == 0:
        peak, peak_kind = peaks()
        upd_ms = passes["update"] / max(nsteps, 1)
        upd_gbs = ALG_BYTES_UPDATE * nloc / (upd_ms * 1e-3) / 1e9
        step_gbs_gpu = ALG_BYTES_STEP * nloc / (ms_step * 1e-3) / 1e9
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_reference_sample()
        line = {
            "metric": METRIC, "value": value, "unit": "params/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_dict(world),
            "hbm_gbs_per_gpu": step_gbs_gpu, "hbm_frac_per_gpu": step_gbs_gpu / peak,
            "alg_bytes_per_param": ALG_BYTES_STEP,
            "passes_ms_per_step": {k: v / max(nsteps, 1) for k, v in passes.items()},
            "roofline": {"kernel": "apply_kernel (update + per-tensor requant)", "bound": "hbm", "achieved": upd_gbs, "peak": peak,
                         "unit": "GB/s", "frac": upd_gbs / peak, "peak_source": peak_kind,
                         "alg_bytes_per_launch": ALG_BYTES_UPDATE * nloc,
                         "traffic": TRAFFIC_BYTES_PER_PARAM_APPLY * nloc,
                         "traffic_source": "ncu capture of an 8-tensor case scaled by params"},
            "e2e": {"value": TOTAL / (e2e_ms * 1e-3), "unit": "params/s", "ms_per_step": e2e_ms,
                    "wall_ms_per_step": wall * 1e3 / args.e2e_steps,
                    "h2d_bytes_per_step": 2 * nloc, "d2h_bytes_per_step": 80},
            "gpu_launches": args.steps * (2 if world == 1 else 3),
            "clocks": clk.summary(),
            "last_step": {k: res[k] for k in ("grad_norm", "clip_coef", "clipped", "skipped", "scale_used")},
        }
        if cb:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
