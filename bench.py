"""Benchmark of the fused mixed-precision step (BASELINE.json metric:
"fused mixed-precision step: params/s & HBM GB/s (% of peak), 1/2/4/8 B200").

Workload (configs[4], the 1B-param flat model the target is quoted on; it
fits one B200): 64 x 4096x4096 float32 master weights ~ N(0, 0.02^2),
bfloat16 gradients ~ N(0, 1e-3^2) x loss scale 4096, AdamW (lr 1e-3, betas
0.9/0.999, eps 1e-8, wd 0.01) + global-norm clip 1.0, NVFP4 requant with a
per-tensor scale.  With N GPUs the 64 tensors are ZeRO-1-sharded (8 whole
tensors per rank at N=8): total work is fixed, scaling is "strong".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload flat1b|resnet18|lenet]

`--workload resnet18` (configs[3], 62 tensors, 11.2 M params, AdamW, BF16
grads, FP8-E4M3 per-tensor) and `--workload lenet` (configs[0], 10 tensors,
61,706 params, SGD-momentum, FP16 grads, FP16 out) are secondary lines: the
same step on the reference's smaller configurations, where launch latency
rather than HBM bandwidth bounds the step.  Their gradients are fixed across
steps (no inf injection), as for the 1B model.

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
WORKLOAD = "flat1b"
QUANT_BYTES = {"none": 0.0, "fp16": 2.0, "bf16": 2.0, "fp8": 1.0, "bf8": 1.0, "fp8_tensor": 1.0,
               "mxfp4": 17 / 32, "nvfp4": 9 / 16, "nvfp4_tensor": 9 / 16}
GRAD_BYTES = {"float32": 4, "float16": 2, "bfloat16": 2}


def alg_bytes_per_param(wl, quant):
    """HBM bytes one parameter needs per step: its gradient read, master and
    optimizer states read and written, and its re-quantised code written."""
    nstates = {"sgd": 1 if wl.hyper.get("momentum", 0.0) > 0 else 0, "adam": 2, "adamw": 2}[wl.optimizer]
    return GRAD_BYTES[wl.grad_dtype] + 8 * (1 + nstates) + QUANT_BYTES[quant]


def make_workload(name, ntensors):
    from odyssey_b200 import workloads as W
    if name == "flat1b":
        return W.flat1b(ntensors=ntensors, side=SIDE)
    wl = W.lenet() if name == "lenet" else W.resnet18()
    wl.inf_every = 0
    return wl


FALLBACK_HBM_GBS = 6650.0
# DRAM bytes per param of one apply_kernel launch, measured with ncu
# (dram__bytes_read.sum + dram__bytes_write.sum of the 8-tensor case
# `--tensors 8`, divided by its 134,217,728 params; traffic grows with the
# params a launch processes)
TRAFFIC_BYTES_PER_PARAM_APPLY = 30.48


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
        import tempfile
        self.f = tempfile.TemporaryFile(mode="w+")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        # the sampler needs a moment to start: wait (at most 5 s) for its
        # first line, so that short timed regions are sampled too
        t0 = time.time()
        while self.p and self.p.poll() is None and time.time() - t0 < 5.0:
            if os.fstat(self.f.fileno()).st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *a):
        if self.p:
            time.sleep(0.25)  # one more sample interval after the timed region
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.seek(0)
        self.out = self.f.read()
        self.f.close()

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


def cpu_reference_sample(seconds=12.0, ntensors=1, quant="nvfp4_tensor", threads=None):
    """The oracle (CPU restatement of the reference path) on the host cores:
    the workload's step (for the 1B model over `ntensors` of its 4096x4096
    tensors; the smaller models whole), repeated for about `seconds`, on all
    host threads or on `threads`."""
    from oracle import oracle as O
    O.build()
    threads = threads or os.cpu_count() or 1
    O.set_threads(threads)
    wl = make_workload(WORKLOAD, ntensors)
    gdt = {"float32": O.F32, "float16": O.F16, "bfloat16": O.BF16}[wl.grad_dtype]
    qk = {"none": 0, "fp16": 1, "bf16": 2, "fp8": 3, "bf8": 4, "fp8_tensor": 5, "mxfp4": 6, "nvfp4": 7,
          "nvfp4_tensor": 8}[quant]
    specs = [{"numel": n, "grad_dtype": gdt, "quant": qk} for n in wl.numels]
    hy = wl.hyper
    opt = {"sgd": O.SGD, "adam": O.ADAM, "adamw": O.ADAMW}[wl.optimizer]
    sk = {k: v for k, v in wl.step_kwargs().items() if k in ("initial_scale", "growth_factor", "backoff_factor",
                                                               "growth_interval", "min_scale", "max_scale")}
    m = O.Model(specs, opt, hy["learning_rate"], momentum=hy.get("momentum", 0.0), beta1=hy.get("beta1", 0.9),
                beta2=hy.get("beta2", 0.999), epsilon=hy.get("epsilon", 1e-8),
                weight_decay=hy.get("weight_decay", 0.0), clip_enabled=wl.clip is not None,
                max_norm=wl.clip or 1.0, scaler_kwargs=sk)
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
    what = (f"{ntensors} x 4096x4096 tensor(s) ({params} params) of the 1B workload" if WORKLOAD == "flat1b"
            else f"the whole {wl.name} model ({params} params)")
    return {"value": params / sec, "unit": "params/s", "cores": threads, "kind": "port",
            "sample": f"{what}, {wl.optimizer}{'+clip' if wl.clip else ''}+{quant}, {len(times)} steps, "
                      f"median {sec * 1e3:.3f} ms/step, {threads} OpenMP threads on {cpu_info()[0]}"}


def with_single_thread(cb, sample):
    """Adds the one-thread figure (the reference's path is single-threaded)
    to an all-threads CPU baseline."""
    cb["single_thread"] = {"value": sample["value"], "unit": sample["unit"], "cores": 1,
                           "sample": sample["sample"]}
    return cb


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cb = cpu_reference_sample(seconds=max(3.0, min(30.0, 2.0 * args.steps)), quant=QUANT)
    with_single_thread(cb, cpu_reference_sample(seconds=8.0, quant=QUANT, threads=1))
    line = {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "params/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": TOTAL / cb["value"] * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_dict(world),
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "params/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- the standalone quantiser -------------------
# name: (kind, side, source dtype, bytes read+written per element by the
# quantiser's kernels: source read (twice with the amax pre-pass of the
# per-tensor scale) + codes written)
QUANT_WORKLOADS = {
    "mxfp4": dict(kind=6, side=4096, sdt="float32", bytes_per_elem=4 + 17 / 32,
                  name="mxfp4_4096x4096_f32_outliers (configs[1])"),
    "nvfp4": dict(kind=8, side=8192, sdt="bfloat16", bytes_per_elem=2 + 2 + 9 / 16,
                  name="nvfp4_tensor_scaled_8192x8192_bf16_outliers (configs[2])"),
    # configs[1] with its scale rule as BASELINE states it (OCP MX v1.0)
    "mxfp4_ocp": dict(kind=9, side=4096, sdt="float32", bytes_per_elem=4 + 17 / 32,
                      name="mxfp4_ocp_4096x4096_f32_outliers (configs[1], OCP MX rule)"),
}
QUANT_METRIC = "standalone quantiser: elements/s & HBM GB/s (% of peak)"


def _quant_input(spec, seed, device):
    """N(0,1) with 0.1 % of positions x100; bfloat16 N(0, 0.02^2)
    with 0.05 % x50; positions drawn without replacement."""
    import torch
    n = spec["side"] ** 2
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if spec["kind"] in (6, 9):
        x = torch.randn(n, device=device, generator=g)
        idx = torch.randperm(n, device=device, generator=g)[: n // 1000]
        x[idx] *= 100.0
        return x
    x = torch.randn(n, device=device, generator=g) * 0.02
    idx = torch.randperm(n, device=device, generator=g)[: n * 5 // 10000]
    x[idx] *= 50.0
    return x.to(torch.bfloat16)


def _quant_cpu_sample(spec, x_host, seconds, threads=None):
    """The oracle's quantiser (all host threads, or `threads`) over the same
    tensor."""
    from oracle import oracle as O
    O.build()
    threads = threads or os.cpu_count() or 1
    O.set_threads(threads)
    if spec["sdt"] == "bfloat16":
        x32 = (x_host.view(np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)
    else:
        x32 = x_host
    out = np.zeros(O.quant_bytes(spec["kind"], x32.size), np.uint8)
    O.lib().ora_quantize(spec["kind"], x32.ctypes.data, x32.size, out.ctypes.data)
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        O.lib().ora_quantize(spec["kind"], x32.ctypes.data, x32.size, out.ctypes.data)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": x32.size / sec, "unit": "elems/s", "cores": threads, "kind": "port",
            "sample": f"the whole tensor ({x32.size} elements), {len(times)} runs, median {sec * 1e3:.1f} ms, "
                      f"{threads} OpenMP threads on {cpu_info()[0]}"}


def run_quant(args):
    """the standalone quantiser on one GPU per rank
    (replicas: each rank quantises its own copy; no collective)."""
    spec = QUANT_WORKLOADS[args.workload]
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    n = spec["side"] ** 2
    config = {"workload": spec["name"], "elements": n, "source_dtype": GDT_SHORT[spec["sdt"]],
              "kind": args.workload + ("_tensor" if spec["kind"] == 8 else ""),
              "parallelism": f"replicas x{world}",
              "l2": "L2 flushed (256 MB read) before every timed launch, outside its events"}
    if args.impl == "reference":
        if rank != 0:
            return 0
        import torch
        x = _quant_input(spec, 7, "cpu")
        xh = (x.view(torch.int16).numpy().view(np.uint16) if spec["sdt"] == "bfloat16" else x.numpy())
        cb = with_single_thread(_quant_cpu_sample(spec, xh, max(3.0, min(30.0, 2.0 * args.steps))),
                                _quant_cpu_sample(spec, xh, 5.0, threads=1))
        print(json.dumps({"metric": QUANT_METRIC, "impl": "reference", "value": cb["value"], "unit": "elems/s",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": n / cb["value"] * 1e3, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                          "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "elems/s",
                                                      "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return 0
    import torch
    import torch.distributed as dist
    from odyssey_b200 import _lib as L
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo")
    kind = spec["kind"]
    x = _quant_input(spec, 7 + rank, "cuda")
    qb = L.quant_bytes(kind, n)
    out = torch.empty(qb, dtype=torch.uint8, device="cuda")
    ts = torch.zeros(1, dtype=torch.float32, device="cuda")
    scratch = torch.zeros(2, dtype=torch.int32, device="cuda")
    # L2 flush by READING 256 MB (a write would leave L2 full of dirty lines
    # whose write-back the next launch would pay for)
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sdt = L.F32 if spec["sdt"] == "float32" else L.BF16
    lib = L.lib()
    scaled = kind == 8

    def launch():
        L.check(lib.ody_quantize_on_stream(kind, x.data_ptr(), sdt, n, out.data_ptr(),
                                           ts.data_ptr() if scaled else None,
                                           scratch.data_ptr() if scaled else None, stream.cuda_stream))

    for _ in range(max(args.warmup, 3)):
        launch()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        # about a second of back-to-back launches while the clock sampler
        # (200 ms period) starts, then the timed launches
        w0 = time.perf_counter()
        while time.perf_counter() - w0 < min(args.clock_warm_s, 1.0):
            for _ in range(50):
                launch()
            torch.cuda.synchronize()
        for e0, e1 in evs:
            flush.sum()
            e0.record(stream)
            launch()
            e1.record(stream)
        torch.cuda.synchronize()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    # end to end through the public API: pinned host source -> device ->
    # quantise -> codes back to pinned host memory, on one stream
    esz = 4 if sdt == L.F32 else 2
    hx = torch.empty(n * esz, dtype=torch.uint8, pin_memory=True)
    hx.copy_(x.view(torch.uint8).cpu())
    hout = torch.empty(qb, dtype=torch.uint8, pin_memory=True)
    xb = x.view(torch.uint8)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for it in range(4):
        if it == 1:
            e0.record(stream)
        xb.copy_(hx, non_blocking=True)
        launch()
        hout.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / 3
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        xh = hx.numpy().view(np.float32 if sdt == L.F32 else np.uint16)
        cb = with_single_thread(_quant_cpu_sample(spec, xh, 12.0), _quant_cpu_sample(spec, xh, 5.0, threads=1))
    if rank == 0:
        peak, peak_kind = peaks()
        gbs = spec["bytes_per_elem"] * n / (ms * 1e-3) / 1e9
        line = {"metric": QUANT_METRIC, "value": world * n / (ms * 1e-3), "unit": "elems/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "roofline": {"kernel": "quantize_kernel" + (" + amax_kernel" if scaled else ""), "bound": "hbm",
                             "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "peak_source": peak_kind, "alg_bytes_per_launch": spec["bytes_per_elem"] * n,
                             "traffic": None},
                "e2e": {"value": world * n / (e2e_ms * 1e-3), "unit": "elems/s", "ms_per_step": e2e_ms,
                        "h2d_bytes_per_step": n * esz, "d2h_bytes_per_step": qb},
                "gpu_launches": args.steps * (2 if scaled else 1), "clocks": clk.summary()}
        if cb:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


GDT_SHORT = {"float32": "f32", "float16": "f16", "bfloat16": "bf16"}
QUANT = "nvfp4_tensor"


def config_dict(world):
    if WORKLOAD != "flat1b":
        wl = make_workload(WORKLOAD, NT)
        return {"workload": wl.name + (" (configs[0])" if WORKLOAD == "lenet" else " (configs[3])"),
                "params": TOTAL, "tensors": len(wl.numels), "grad_dtype": GDT_SHORT[wl.grad_dtype],
                "master_dtype": "f32", "optimizer": wl.optimizer, "clip_max_norm": wl.clip, "quant": QUANT,
                "loss_scale": wl.loss_scale, "parallelism": f"zero1 whole-tensor shards x{world}",
                "l2": "model smaller than L2; no flush (secondary, latency-bound line)"}
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
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--e2e-serial", action="store_true",
                    help="e2e without double-buffered gradients (each upload waits for the previous step)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tensors", type=int, default=64,
                    help="number of 4096x4096 tensors (64 = the 1B workload; fewer only for profiling)")
    ap.add_argument("--quant", default=None,
                    help="re-quantisation kind (default: the workload's own; others only for comparisons)")
    ap.add_argument("--clock-warm-s", type=float, default=1.5,
                    help="untimed steps run for about this long while the clock sampler starts (0 for ncu captures)")
    ap.add_argument("--graph", default="auto", choices=["auto", "on", "off"],
                    help="replay each step as one CUDA graph launch (auto: on with one GPU)")
    ap.add_argument("--dp", default="none", choices=["none", "fused", "nccl"],
                    help="data-parallel gradients: every rank holds full-model gradients and each step first "
                         "reduce-scatters them, fused with pass 1 (fused) or by ncclReduceScatter (nccl, "
                         "for comparison); none = gradients already reduced (the headline)")
    ap.add_argument("--workload", default="flat1b", choices=["flat1b", "resnet18", "lenet", "mxfp4", "nvfp4", "mxfp4_ocp"],
                    help="flat1b = the headline 1B model; resnet18 / lenet = secondary step lines; mxfp4 / "
                         "nvfp4 = the standalone quantiser on configs[1] / configs[2]")
    ap.add_argument("--placement", default="auto", choices=["auto", "interleaved", "at_end"],
                    help="where the apply kernel runs the per-tensor-scaled requant jobs (results identical)")
    args = ap.parse_args()
    if args.workload in QUANT_WORKLOADS:
        return run_quant(args)
    global NT, TOTAL, WORKLOAD, QUANT, ALG_BYTES_STEP, ALG_BYTES_UPDATE
    WORKLOAD, NT = args.workload, args.tensors
    wl = make_workload(WORKLOAD, NT)
    QUANT = args.quant or wl.quant
    TOTAL = wl.total
    ALG_BYTES_STEP = ALG_BYTES_UPDATE = alg_bytes_per_param(wl, QUANT)
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    import odyssey_b200 as ody
    from odyssey_b200 import _lib as L

    torch.cuda.set_device(local)
    if world > 1:
        # host-side plumbing only (NCCL id broadcast, barriers, max over ranks);
        # the step's own exchange runs on the library's NCCL communicator
        dist.init_process_group("gloo")
    kw = wl.step_kwargs()
    kw["device"] = local
    kw["quant"] = QUANT
    kw["requant_placement"] = args.placement
    if world > 1:
        ctx = ody.MixedPrecisionStep.from_process_group(wl.numels, **kw)
    else:
        ctx = ody.MixedPrecisionStep(wl.numels, **kw)
    use_graph = args.graph == "on" or (args.graph == "auto" and world == 1)
    if use_graph:
        ctx.set_graph(True)
    owned = ctx.owned
    nloc = sum(wl.numels[i] for i in owned)
    gdt = getattr(torch, wl.grad_dtype)
    gsz = GRAD_BYTES[wl.grad_dtype]

    # synthetic inputs generated on the device (seeded), copied into the arenas
    gen = torch.Generator(device="cuda")
    for i in owned:
        n = wl.numels[i]
        gen.manual_seed(1000 + i)
        m = torch.randn(n, device="cuda", generator=gen) * wl.master_std
        ctx.upload(L.BUF_MASTER, i, m)
        gen.manual_seed(5000 + i)
        g = (torch.randn(n, device="cuda", generator=gen) * (wl.grad_std * wl.loss_scale)).to(gdt)
        ctx.upload(L.BUF_GRAD, i, g)
        del m, g
    torch.cuda.synchronize()

    # data-parallel gradients: each rank's own full-model gradients (seeded
    # per rank), reduce-scattered inside the timed step
    rs_step = None
    if args.dp != "none":
        if args.dp == "fused":
            ctx.dp_attach()
        full = torch.empty(sum((n + 63) // 64 * 64 for n in wl.numels), dtype=gdt, device="cuda")
        off = 0
        for i, n in enumerate(wl.numels):
            gen.manual_seed(5000 + i + 100000 * rank)
            g = (torch.randn(n, device="cuda", generator=gen) * (wl.grad_std * wl.loss_scale)).to(gdt)
            if args.dp == "fused":
                ctx.upload(L.BUF_DP_GRAD, i, g)
            else:
                full[off:off + n].copy_(g)
            off += (n + 63) // 64 * 64
            del g
        if args.dp == "fused":
            del full
        else:
            # ncclReduceScatter of the full buffer straight into this rank's
            # gradient arena (equal shards only), ordered on the step's stream
            if any(wl.numels[i] % 64 for i in range(len(wl.numels))) or len(wl.numels) % world:
                raise SystemExit("--dp nccl needs equal, unpadded shards")
            nccl_pg = dist.new_group(backend="nccl") if world > 1 else None

            class _Arena:
                def __init__(self, ptr, n):
                    self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False),
                                                     "version": 3}

            arena = torch.as_tensor(_Arena(ctx.device_ptr(L.BUF_GRAD, owned[0]), nloc), device="cuda")
            arena = arena.view(gdt)
            rs_stream = torch.cuda.ExternalStream(ctx.stream_handle())

            def rs_step():
                with torch.cuda.stream(rs_stream):
                    if world > 1:
                        dist.reduce_scatter_tensor(arena, full, group=nccl_pg)
                    else:
                        arena.copy_(full)
        torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    t = 1
    w0 = time.perf_counter()
    for _ in range(args.warmup):
        if rs_step:
            rs_step()
        ctx.step(t)
        t += 1
    # every rank must run the same number of steps (each step has a
    # collective): the untimed clock-warm-up count is agreed from the slowest
    # rank's warm-up time
    per_step = torch.tensor([(time.perf_counter() - w0) / max(args.warmup, 1)], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(per_step, op=dist.ReduceOp.MAX)
    n_clock_warm = max(3, min(5000, int(args.clock_warm_s / max(per_step.item(), 1e-6))))
    stream = torch.cuda.ExternalStream(ctx.stream_handle())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with Clocks(local) as clk:
        # keep the GPU loaded while the clock sampler starts (untimed steps);
        # per-pass times are taken here, so that the timed steps carry no
        # extra events
        ctx.set_timing(True)
        ctx.pass_times()
        for _ in range(n_clock_warm):
            if rs_step:
                rs_step()
            ctx.step_async(t)
            t += 1
            ctx.wait()
        passes, nsteps = ctx.pass_times()
        ctx.set_timing(False)
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            if rs_step:
                rs_step()
            ctx.step_async(t)
            t += 1
        ev1.record(stream)
        res = ctx.wait()
        ev1.synchronize()
    barrier()
    ms_total = ev0.elapsed_time(ev1)
    # each rank's own pass times (per step), taken over the same untimed
    # window: the exchange of a rank that finished its stats pass early
    # includes its wait for the slowest rank
    keys = ("stats", "exchange", "update")
    mine = torch.tensor([passes[k] / max(nsteps, 1) for k in keys], dtype=torch.float64)
    per_rank = [mine.tolist()]
    if world > 1:
        allp = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allp, mine)
        per_rank = [p.tolist() for p in allp]
        x = torch.tensor([ms_total, passes["update"], passes["stats"], passes["requant"], passes["exchange"]],
                         dtype=torch.float64)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        ms_total, passes["update"], passes["stats"], passes["requant"], passes["exchange"] = x.tolist()
    ms_step = ms_total / args.steps
    value = TOTAL / (ms_step * 1e-3)

    # ---- end to end through the C ABI: pinned host gradients -> step -> result
    # (data-parallel: this rank's full-model gradients; not measured for the
    # NCCL comparison mode)
    e2e_ms = wall = None
    e2e_idx = owned if args.dp == "none" else list(range(len(wl.numels)))
    e2e_buf = L.BUF_GRAD if args.dp == "none" else L.BUF_DP_GRAD
    h2d_bytes = gsz * sum(wl.numels[i] for i in e2e_idx)
    if args.dp != "nccl":
        pinned = [torch.empty(wl.numels[i] * gsz, dtype=torch.uint8, pin_memory=True) for i in e2e_idx]
        for k, i in enumerate(e2e_idx):
            pinned[k].copy_(torch.from_numpy(ctx.download(e2e_buf, i).view(np.uint8)))
        lib = L.lib()

        def upload_all():
            for k, i in enumerate(e2e_idx):
                L.check(lib.ody_upload_async(ctx._ctx, e2e_buf, i, pinned[k].data_ptr(), pinned[k].numel()),
                        ctx._ctx)

        # double-buffered gradient arenas (not with data-parallel gradients):
        # step t+1's upload is queued right after step t, on a copy stream,
        # so the PCIe copy overlaps step t's kernels
        dbuf = args.dp == "none" and not args.e2e_serial
        if dbuf:
            ctx.set_grad_double_buffer(True)
        upload_all()
        ctx.step(t)
        t += 1
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        e0.record(stream)
        if dbuf:
            upload_all()
            for k in range(args.e2e_steps):
                ctx.step_async(t)
                t += 1
                if k + 1 < args.e2e_steps:
                    upload_all()  # the next step's gradients, while this step runs
                ctx.wait()  # the device->host read of this step's result
        else:
            for _ in range(args.e2e_steps):
                upload_all()
                ctx.step(t)  # synchronous: includes the device->host read of the step result
                t += 1
        e1.record(stream)
        e1.synchronize()
        wall = time.perf_counter() - w0
        if dbuf:
            ctx.set_grad_double_buffer(False)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            x = torch.tensor([e2e_ms], dtype=torch.float64)
            dist.all_reduce(x, op=dist.ReduceOp.MAX)
            e2e_ms = x.item()

    # N > 1: the all-gather of the re-quantised model after the sharded step
    # (not part of the step; reported beside it)
    gather = None
    if world > 1:
        gq_total = ctx.quant_layout()[2]
        ctx.gather_quant()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(5):
            ctx.gather_quant()
        g1.record(stream)
        g1.synchronize()
        x = torch.tensor([g0.elapsed_time(g1) / 5], dtype=torch.float64)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        gather = {"ms": x.item(), "bytes": gq_total, "gbs": gq_total / (x.item() * 1e-3) / 1e9}

    if rank == 0:
        peak, peak_kind = peaks()
        upd_ms = passes["update"] / max(nsteps, 1)
        upd_gbs = ALG_BYTES_UPDATE * nloc / (upd_ms * 1e-3) / 1e9
        step_gbs_gpu = ALG_BYTES_STEP * nloc / (ms_step * 1e-3) / 1e9
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            cb = with_single_thread(cpu_reference_sample(quant=QUANT),
                                    cpu_reference_sample(seconds=8.0, quant=QUANT, threads=1))
        line = {
            "metric": METRIC, "value": value, "unit": "params/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_dict(world),
            "hbm_gbs_per_gpu": step_gbs_gpu, "hbm_frac_per_gpu": step_gbs_gpu / peak,
            "alg_bytes_per_param": ALG_BYTES_STEP,
            "passes_ms_per_step": {k: v / max(nsteps, 1) for k, v in passes.items()},
            "passes_ms_per_rank": {k: [r[j] for r in per_rank] for j, k in enumerate(keys)},
            "requant_placement": args.placement,
            "roofline": {"kernel": "apply_kernel (update + per-tensor requant)", "bound": "hbm", "achieved": upd_gbs, "peak": peak,
                         "unit": "GB/s", "frac": upd_gbs / peak, "peak_source": peak_kind,
                         "alg_bytes_per_launch": ALG_BYTES_UPDATE * nloc,
                         "traffic": (TRAFFIC_BYTES_PER_PARAM_APPLY * nloc
                                     if WORKLOAD == "flat1b" and QUANT == "nvfp4_tensor" else None),
                         "traffic_source": ("ncu capture of an 8-tensor case scaled by params"
                                            if WORKLOAD == "flat1b" and QUANT == "nvfp4_tensor" else None)},
            "e2e": None if e2e_ms is None else {
                "value": TOTAL / (e2e_ms * 1e-3), "unit": "params/s", "ms_per_step": e2e_ms,
                "wall_ms_per_step": wall * 1e3 / args.e2e_steps,
                "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": 80,
                "overlap": "double-buffered gradients" if (args.dp == "none" and not args.e2e_serial) else "none",
                "outputs": "the step result (80 B) is read back every step; master weights, states and the "
                           "re-quantised weights stay in device memory for the next forward pass"},
            "gpu_launches": args.steps * (2 if world == 1 else 3),
            "graph_mode": use_graph,
            "dp_gradients": args.dp,
            "clocks": clk.summary(),
            "last_step": {k: res[k] for k in ("grad_norm", "clip_coef", "clipped", "skipped", "scale_used")},
        }
        if cb:
            line["cpu_baseline"] = cb
        if gather:
            line["gather_quant"] = gather
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
