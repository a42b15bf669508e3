"""GPU parity of the fused step (MixedPrecisionStep -> ody_step) against the
oracle's restatement of the reference call sequence: master weights and
optimizer states within 2 float32 ulp (they come out bit-identical), quantised
codes and scales bit-exact, skip/backoff decisions identical."""
import numpy as np
import pytest

from odyssey_b200 import workloads as W

pytestmark = pytest.mark.gpu

GDT = {"float32": 0, "float16": 1, "bfloat16": 2}
OPT = {"sgd": 0, "adam": 1, "adamw": 2, "lion": 3, "rmsprop": 4, "adagrad": 5}
QK = {"none": 0, "fp16": 1, "bf16": 2, "fp8": 3, "bf8": 4, "fp8_tensor": 5, "mxfp4": 6, "nvfp4": 7,
      "nvfp4_tensor": 8}


def ulp_diff(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


def run_pair(oracle, wl, nsteps, numels=None, quants=None, seed=0, t0=1, check_every=1, ctx_kwargs=None):
    """Run the same workload through the GPU context and the oracle."""
    from odyssey_b200 import MixedPrecisionStep
    numels = numels or wl.numels
    kw = wl.step_kwargs()
    if quants is not None:
        kw["quant"] = quants
    qlist = kw["quant"] if isinstance(kw["quant"], list) else [kw["quant"]] * len(numels)
    ctx = MixedPrecisionStep(numels, **kw, **(ctx_kwargs or {}))
    specs = [{"numel": n, "grad_dtype": GDT[wl.grad_dtype], "quant": QK[q]} for n, q in zip(numels, qlist)]
    hy = wl.hyper
    sk = {k: kw[k] for k in ("initial_scale", "growth_factor", "backoff_factor", "growth_interval", "min_scale",
                             "max_scale") if k in kw}
    model = oracle.Model(specs, OPT[wl.optimizer], hy["learning_rate"], momentum=hy.get("momentum", 0.0),
                         beta1=hy.get("beta1", 0.9), beta2=hy.get("beta2", 0.999), epsilon=hy.get("epsilon", 1e-8),
                         weight_decay=hy.get("weight_decay", 0.0), clip_enabled=wl.clip is not None,
                         max_norm=wl.clip or 1.0, scaler_kwargs=sk, alpha=hy.get("alpha", 0.99))
    master = wl.master(seed, numels)
    for i, m in enumerate(master):
        ctx.set_master(i, m)
        model.master[i][:] = m
    t = t0
    results = []
    for s in range(nsteps):
        grads = wl.grads(s, seed + 1, numels)
        for i, g in enumerate(grads):
            ctx.set_grad(i, g)
        r = ctx.step(t)
        ro = model.step(grads, t)
        results.append((r, ro))
        assert r["skipped"] == ro.skipped, s
        assert r["nonfinite_count"] == ro.nonfinite, s
        assert r["scale_used"] == ro.scale_used and r["scale_next"] == ro.scale_next, s
        assert r["step_count"] == ro.step_count and r["overflow_count"] == ro.overflow_count
        assert r["clipped"] == ro.clipped, s
        if np.isfinite(ro.sumsq):
            assert abs(r["sumsq"] - ro.sumsq) <= 1e-12 * max(ro.sumsq, 1e-300), s
            assert r["grad_norm"] == ro.norm and r["clip_coef"] == ro.coef, s
        else:
            assert not np.isfinite(r["sumsq"]), s
        if not r["skipped"] and wl.optimizer in ("adam", "adamw", "rmsprop"):
            t += 1
        if (s + 1) % check_every == 0 or s == nsteps - 1:
            compare_state(ctx, model, numels, qlist, wl.optimizer)
    return ctx, model, results


def compare_state(ctx, model, numels, qlist, optimizer):
    for i in range(len(numels)):
        d = ulp_diff(ctx.master(i), model.master[i])
        assert d.max() <= 2, (i, d.max())
        if optimizer != "sgd" or model.cfg.momentum > 0:
            assert ulp_diff(ctx.state(i, 0), model.s1[i]).max() <= 2, i
        if optimizer in ("adam", "adamw") or (optimizer == "rmsprop" and model.cfg.momentum > 0):
            assert ulp_diff(ctx.state(i, 1), model.s2[i]).max() <= 2, i
        if QK[qlist[i]] != 0:
            q = ctx.get_quant(i)
            nb = q.data.size
            np.testing.assert_array_equal(q.data, model.qout[i][:nb], err_msg=f"tensor {i}")
            assert np.float32(q.tensor_scale) == model.qscale[i][0]


def test_lenet_sgd_fp16_100_steps(oracle):
    """Config 1 at full size: 100 steps, seed 0, FP16 grads x 1024."""
    ctx, model, res = run_pair(oracle, W.lenet(), 100, check_every=25)
    ctx.close()


def test_lenet_with_overflow_steps(oracle):
    wl = W.lenet()
    wl.inf_every = 3
    ctx, model, res = run_pair(oracle, wl, 10)
    assert sum(r["skipped"] for r, _ in res) == 3
    ctx.close()


def test_resnet18_adamw_fp8_tensor(oracle):
    """Config 4 at full size (62 tensors), with the inf injection every 100th
    step exercised by a shortened interval."""
    wl = W.resnet18()
    wl.inf_every = 4
    ctx, model, res = run_pair(oracle, wl, 9, check_every=3)
    assert [r["skipped"] for r, _ in res] == [0, 0, 0, 0, 1, 0, 0, 0, 1]
    ctx.close()


def test_flat_adamw_clip_nvfp4_tensor_small(oracle):
    """Config 5's path (AdamW + global-norm clip + NVFP4 per-tensor scale) on
    4 tensors of 512x512."""
    wl = W.flat1b(ntensors=4, side=512)
    ctx, model, res = run_pair(oracle, wl, 4)
    assert all(r["clipped"] for r, _ in res)
    ctx.close()


HYPER = {
    "sgd": dict(learning_rate=1e-2, momentum=0.9, weight_decay=0.01),
    "adam": dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01),
    "adamw": dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01),
    "lion": dict(learning_rate=1e-4, beta1=0.9, beta2=0.99, weight_decay=0.01),
    "rmsprop": dict(learning_rate=1e-2, alpha=0.9, epsilon=1e-8, weight_decay=0.01, momentum=0.9),
    "adagrad": dict(learning_rate=1e-2, epsilon=1e-10, weight_decay=0.01),
}


@pytest.mark.parametrize("opt", ["sgd", "adam", "adamw", "lion", "rmsprop", "adagrad"])
@pytest.mark.parametrize("gdt", ["float32", "float16", "bfloat16"])
def test_all_kinds_all_optimizers(oracle, opt, gdt):
    """Every re-quantisation kind in one model, ragged tensor sizes."""
    wl = W.Workload("mix", [(1,), (15,), (33,), (2049,), (5000,), (16384 + 64,), (40000,), (7,), (100,)],
                    gdt, "none", opt, HYPER[opt], 0.05, 1e-3, 256.0, clip=0.05)
    quants = ["fp16", "bf16", "fp8", "bf8", "fp8_tensor", "mxfp4", "nvfp4", "nvfp4_tensor", "none"]
    ctx, model, res = run_pair(oracle, wl, 3, quants=quants)
    ctx.close()


def test_rmsprop_without_momentum_fused(oracle):
    """RMSprop without momentum keeps a single state buffer."""
    wl = W.Workload("rms", [(3000,), (70,)], "bfloat16", "nvfp4_tensor", "rmsprop",
                    dict(learning_rate=1e-3, alpha=0.99, epsilon=1e-8), 0.05, 1e-3, 1024.0)
    ctx, model, res = run_pair(oracle, wl, 3)
    ctx.close()


def test_no_scaler_no_clip(oracle):
    wl = W.Workload("plain", [(3000,), (77,)], "float32", "mxfp4", "adam",
                    dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.0),
                    0.05, 1e-3, 1.0)
    from odyssey_b200 import MixedPrecisionStep
    kw = wl.step_kwargs()
    kw["use_gradient_scaler"] = False
    ctx = MixedPrecisionStep(wl.numels, **kw)
    specs = [{"numel": n, "grad_dtype": 0, "quant": 6} for n in wl.numels]
    model = oracle.Model(specs, 1, 1e-3, use_scaler=False, scaler_kwargs={"initial_scale": 1.0})
    for i, m in enumerate(wl.master(0)):
        ctx.set_master(i, m)
        model.master[i][:] = m
    for s in range(3):
        g = wl.grads(s)
        for i, x in enumerate(g):
            ctx.set_grad(i, x)
        r = ctx.step(s + 1)
        ro = model.step(g, s + 1)
        assert r["scale_used"] == ro.scale_used
    compare_state(ctx, model, wl.numels, ["mxfp4"] * 2, "adam")
    ctx.close()


def test_checkpoint_resume_bit_identical(oracle):
    """Export mid-run, continue, import, replay: identical to uninterrupted."""
    from odyssey_b200 import MixedPrecisionStep
    wl = W.flat1b(ntensors=3, side=256)
    kw = wl.step_kwargs()
    ctx = MixedPrecisionStep(wl.numels, **kw)
    for i, m in enumerate(wl.master(0)):
        ctx.set_master(i, m)

    def run(steps, t0):
        for s in steps:
            for i, g in enumerate(wl.grads(s)):
                ctx.set_grad(i, g)
            ctx.step(t0 + s)

    run(range(2), 1)
    blob = ctx.export_state()
    run(range(2, 5), 1)
    final = [ctx.master(i) for i in range(3)]
    codes = [ctx.get_quant(i).data for i in range(3)]
    ctx.import_state(blob)
    run(range(2, 5), 1)
    for i in range(3):
        np.testing.assert_array_equal(ctx.master(i), final[i])
        np.testing.assert_array_equal(ctx.get_quant(i).data, codes[i])
    ctx.close()


def test_step_errors():
    from odyssey_b200 import MixedPrecisionStep, OdysseyError
    ctx = MixedPrecisionStep([100], grad_dtype="float32", optimizer="adamw")
    with pytest.raises(OdysseyError, match="Timestep t must be positive"):
        ctx.step(0)
    with pytest.raises(OdysseyError, match="size mismatch"):
        ctx.set_master(0, np.zeros(99, np.float32))
    ctx.close()


def test_async_pipeline_matches_sync(oracle):
    """ody_step_async + ody_upload_async (pinned host) gives the same state as
    synchronous steps."""
    from odyssey_b200 import MixedPrecisionStep
    wl = W.flat1b(ntensors=2, side=512)
    a = MixedPrecisionStep(wl.numels, **wl.step_kwargs())
    b = MixedPrecisionStep(wl.numels, **wl.step_kwargs())
    for i, m in enumerate(wl.master(0)):
        a.set_master(i, m)
        b.set_master(i, m)
    for s in range(3):
        gs = wl.grads(s)
        for i, g in enumerate(gs):
            a.set_grad(i, g)
            b.set_grad(i, g, sync=False)
        a.step(s + 1)
        b.step_async(s + 1)
        b.wait()
    for i in range(2):
        np.testing.assert_array_equal(a.master(i), b.master(i))
    a.close()
    b.close()


def test_gather_quant_single_rank(oracle):
    """With one rank the gathered model is the local quantised arena in
    global tensor order."""
    wl = W.Workload("gq", [(1000,), (33,), (70000,)], "bfloat16", "none", "adamw",
                    dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01),
                    0.05, 1e-3, 1024.0)
    ctx, model, _ = run_pair(oracle, wl, 2, quants=["nvfp4_tensor", "mxfp4", "fp8_tensor"])
    buf, scales = ctx.gather_quant()
    g = buf.cpu().numpy()
    for i in range(3):
        off, nb, total = ctx.quant_layout(i)
        assert off % 256 == 0 and off + nb <= total
        np.testing.assert_array_equal(g[off:off + nb], model.qout[i][:nb])
        assert scales[i].item() == model.qscale[i][0]
    ctx.close()


def _wide_master(rng, n, lo_exp, hi_exp, zeros=0.02, specials=()):
    """float32 values with log-uniform magnitudes 2^[lo_exp, hi_exp), random
    signs, some exact zeros and the given special values at random places."""
    e = rng.uniform(lo_exp, hi_exp, n)
    x = (np.exp2(e) * rng.choice([-1.0, 1.0], n)).astype(np.float32)
    x[rng.random(n) < zeros] = 0.0
    for v in specials:
        x[rng.integers(n)] = v
    return x


@pytest.mark.parametrize("quant", ["nvfp4_tensor", "nvfp4", "mxfp4"])
def test_nvfp4_tensor_scale_sweep(oracle, quant):
    """FP4 requant of tensors whose scales span the float range (subnormal to
    huge amax, wide in-tensor spread, signed zeros, NaN and Inf elements)
    against the oracle's element-by-element division, bit for bit: NVFP4
    with a per-tensor scale (the requant jobs), and plain NVFP4 / MXFP4
    (encoded inside the update jobs).  SGD with lr 0 keeps the masters as
    written."""
    from odyssey_b200 import MixedPrecisionStep
    rng = np.random.Generator(np.random.PCG64(77))
    ranges = [(-149, -126), (-140, -100), (-60, -20), (-30, 0), (-8, -2), (-2, 2), (0, 30), (20, 60),
              (90, 127), (100, 127.9), (-149, 127.9)]
    masters = []
    for lo, hi in ranges:
        masters.append(_wide_master(rng, 4096 + int(rng.integers(0, 300)), lo, hi))
    masters.append(_wide_master(rng, 3000, -10, 0, specials=[np.nan]))
    masters.append(_wide_master(rng, 3000, -10, 0, specials=[-np.inf]))
    masters.append(_wide_master(rng, 3000, -10, 0, specials=[np.float32(3.4e38), -0.0]))
    masters.append(np.zeros(100, np.float32))
    numels = [m.size for m in masters]
    ctx = MixedPrecisionStep(numels, grad_dtype="float32", quant=quant, optimizer="sgd",
                             learning_rate=0.0, momentum=0.0, weight_decay=0.0, use_gradient_scaler=False)
    specs = [{"numel": n, "grad_dtype": 0, "quant": QK[quant]} for n in numels]
    model = oracle.Model(specs, OPT["sgd"], 0.0, use_scaler=False, scaler_kwargs={"initial_scale": 1.0})
    for i, m in enumerate(masters):
        ctx.set_master(i, m)
        model.master[i][:] = m
    grads = [np.zeros(n, np.float32) for n in numels]
    for i, g in enumerate(grads):
        ctx.set_grad(i, g)
    ctx.step(1)
    model.step(grads, 1)
    for i in range(len(numels)):
        q = ctx.get_quant(i)
        np.testing.assert_array_equal(q.data, model.qout[i][:q.data.size], err_msg=f"tensor {i} {ranges[i:i+1]}")
        if quant == "nvfp4_tensor":
            assert np.float32(q.tensor_scale) == model.qscale[i][0] or (
                np.isnan(q.tensor_scale) and np.isnan(model.qscale[i][0])), i
    ctx.close()


@pytest.mark.parametrize("which", ["lenet", "resnet18"])
def test_graph_mode_matches_eager(oracle, which):
    """Graph mode (one graph launch per step, optimizer constants updated in
    the instantiated graph) gives bit-identical state and decisions to the
    eager path, across skipped steps and a changing Adam timestep."""
    from odyssey_b200 import MixedPrecisionStep
    wl = W.lenet() if which == "lenet" else W.resnet18()
    wl.inf_every = 3
    kw = wl.step_kwargs()
    a = MixedPrecisionStep(wl.numels, **kw)
    b = MixedPrecisionStep(wl.numels, **kw)
    b.set_graph(True)
    for i, m in enumerate(wl.master(0)):
        a.set_master(i, m)
        b.set_master(i, m)
    t = 1
    for s in range(7):
        for i, g in enumerate(wl.grads(s)):
            a.set_grad(i, g)
            b.set_grad(i, g)
        ra, rb = a.step(t), b.step(t)
        assert ra == rb, s
        if not ra["skipped"]:
            t += 1
    for i in range(len(wl.numels)):
        np.testing.assert_array_equal(a.master(i), b.master(i))
        np.testing.assert_array_equal(a.get_quant(i).data, b.get_quant(i).data)
    b.set_graph(False)
    a.close()
    b.close()


@pytest.mark.parametrize("graph", [False, True])
def test_dp_single_rank_matches_plain(oracle, graph):
    """Data-parallel gradients on one rank: the fused reduce-scatter + pass 1
    reads the full-model buffer and must give exactly the plain step (a sum
    over one rank is the gradient itself)."""
    from odyssey_b200 import MixedPrecisionStep
    wl = W.resnet18()
    wl.inf_every = 3
    kw = wl.step_kwargs()
    a = MixedPrecisionStep(wl.numels, **kw)
    b = MixedPrecisionStep(wl.numels, **kw)
    b.set_graph(graph)
    b.dp_attach()
    for i, m in enumerate(wl.master(0)):
        a.set_master(i, m)
        b.set_master(i, m)
    t = 1
    for s in range(5):
        for i, g in enumerate(wl.grads(s)):
            a.set_grad(i, g)
            b.set_dp_grad(i, g)
        ra, rb = a.step(t), b.step(t)
        assert ra == rb, s
        if not ra["skipped"]:
            t += 1
    for i in range(len(wl.numels)):
        np.testing.assert_array_equal(a.master(i), b.master(i))
        np.testing.assert_array_equal(a.download(3, i), b.download(3, i))  # reduced gradients
        np.testing.assert_array_equal(a.get_quant(i).data, b.get_quant(i).data)
    a.close()
    b.close()


def test_reference_checkpoint_layout_resume(oracle, tmp_path):
    """Save a running context in the reference's checkpoint layout, load it
    into a fresh context, and continue: identical to the uninterrupted run."""
    from odyssey_b200 import MixedPrecisionStep
    from odyssey_b200 import checkpoint as ck
    wl = W.resnet18()
    kw = wl.step_kwargs()
    names = [f"p{i}" for i in range(len(wl.numels))]
    a = MixedPrecisionStep(wl.numels, **kw)
    for i, m in enumerate(wl.master(0)):
        a.set_master(i, m)

    def run(ctx, steps, t0):
        for s in steps:
            for i, g in enumerate(wl.grads(s)):
                ctx.set_grad(i, g)
            ctx.step(t0 + s)

    run(a, range(2), 1)
    ck.save_checkpoint(a, str(tmp_path), names, wl.shapes, epoch=1, step=2)
    b = MixedPrecisionStep(wl.numels, **kw)
    assert ck.load_checkpoint(b, str(tmp_path), names) == (1, 2)
    assert b.scaler_state == a.scaler_state
    run(a, range(2, 4), 1)
    run(b, range(2, 4), 1)
    for i in range(len(wl.numels)):
        np.testing.assert_array_equal(a.master(i), b.master(i))
        np.testing.assert_array_equal(a.get_quant(i).data, b.get_quant(i).data)
    a.close()
    b.close()


def test_dp_attach_errors():
    """Data-parallel gradients: a second attach is refused, and the buffer
    kind is refused before an attach."""
    from odyssey_b200 import MixedPrecisionStep, OdysseyError
    from odyssey_b200 import _lib as L
    ctx = MixedPrecisionStep([100, 37], grad_dtype="bfloat16", optimizer="adamw")
    with pytest.raises(OdysseyError, match="not attached"):
        ctx.set_dp_grad(0, np.zeros(100, np.uint16))
    ctx.dp_attach()
    with pytest.raises(OdysseyError, match="already attached"):
        ctx.dp_attach()
    ctx.set_dp_grad(1, np.ones(37, np.uint16))
    np.testing.assert_array_equal(ctx.download(L.BUF_DP_GRAD, 1), np.ones(37, np.uint16))
    ctx.close()


@pytest.mark.parametrize("chunk", [65536, 8192])
def test_long_chunks(oracle, chunk):
    """Apply jobs of the longest chunk length the 1B model uses (65,536
    elements; the size rule gives test-sized models short chunks), with a
    ragged last chunk, against the oracle."""
    wl = W.Workload("long", [(200000,), (65536 * 2,), (70000,)], "bfloat16", "nvfp4_tensor", "adamw",
                    dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01),
                    0.02, 1e-3, 4096.0, clip=1.0)
    ctx, model, res = run_pair(oracle, wl, 3, quants=["nvfp4_tensor", "mxfp4", "fp8_tensor"],
                               ctx_kwargs={"chunk_elems": chunk})
    ctx.close()


@pytest.mark.parametrize("graph", [False, True])
def test_double_buffered_gradients(oracle, graph):
    """Double-buffered gradient arenas: step t+1's gradients uploaded (async,
    copy stream) while step t runs give the oracle's results step by step,
    with an inf step in between; turning it off keeps the staged arena."""
    from odyssey_b200 import MixedPrecisionStep
    wl = W.flat1b(ntensors=3, side=384)
    wl.inf_every = 3
    kw = wl.step_kwargs()
    ctx = MixedPrecisionStep(wl.numels, **kw)
    ctx.set_graph(graph)  # ignored while double-buffering
    specs = [{"numel": n, "grad_dtype": GDT[wl.grad_dtype], "quant": QK[wl.quant]} for n in wl.numels]
    hy = wl.hyper
    model = oracle.Model(specs, OPT[wl.optimizer], hy["learning_rate"], beta1=hy["beta1"], beta2=hy["beta2"],
                         epsilon=hy["epsilon"], weight_decay=hy["weight_decay"], clip_enabled=True,
                         max_norm=wl.clip, scaler_kwargs={"initial_scale": kw["initial_scale"]})
    for i, m in enumerate(wl.master(0)):
        ctx.set_master(i, m)
        model.master[i][:] = m
    t = to = 1
    if graph:
        # two captured-graph steps first, so that a graph naming the single
        # arena exists when double-buffering starts (it must not be replayed)
        for s0 in (100, 101):
            g0 = wl.grads(s0)
            for i, g in enumerate(g0):
                ctx.set_grad(i, g)
            r = ctx.step(t)
            ro = model.step(g0, to)
            assert r["clip_coef"] == ro.coef
            t += 1
            to += 1
    ctx.set_grad_double_buffer(True)
    nsteps = 7
    grads = [wl.grads(s) for s in range(nsteps + 1)]
    kept = []  # the host arrays must outlive their async copies
    for i, g in enumerate(grads[0]):
        kept.append(ctx.set_grad(i, g, sync=False))
    for s in range(nsteps):
        ctx.step_async(t)
        for i, g in enumerate(grads[s + 1]):
            kept.append(ctx.set_grad(i, g, sync=False))
        r = ctx.wait()
        ro = model.step(grads[s], to)
        assert r["skipped"] == ro.skipped and r["clip_coef"] == ro.coef and r["scale_next"] == ro.scale_next, s
        if not r["skipped"]:
            t += 1
            to += 1
    compare_state(ctx, model, wl.numels, [wl.quant] * len(wl.numels), wl.optimizer)
    # off: the arena staged for the next step (grads[nsteps]) is the one kept
    ctx.set_grad_double_buffer(False)
    r = ctx.step(t)
    ro = model.step(grads[nsteps], to)
    assert r["skipped"] == ro.skipped and r["clip_coef"] == ro.coef
    if not r["skipped"]:
        t += 1
        to += 1
    # and single-arena steps afterwards (in graph mode: a fresh capture)
    for s0 in (200, 201):
        g0 = wl.grads(s0)
        for i, g in enumerate(g0):
            ctx.set_grad(i, g)
        r = ctx.step(t)
        ro = model.step(g0, to)
        assert r["skipped"] == ro.skipped and r["clip_coef"] == ro.coef
        t += 1
        to += 1
    compare_state(ctx, model, wl.numels, [wl.quant] * len(wl.numels), wl.optimizer)
    ctx.close()


def test_resnet18_adamw_fp8_tensor_1000_steps(oracle):
    """Config 4 at its stated length: 1,000 AdamW steps (numbered 1..1000) on
    ResNet-18 with an inf injected on every 100th step, FP8-E4M3 per-tensor
    requant, against the oracle (state compared every 100 steps).  Exactly
    the 10 inf steps are skipped, each backs the scale off by half, and the
    step / overflow counters match (the reference's overflow-recovery
    sequence, test_multi_precision_training.mojo:141-177)."""
    from odyssey_b200 import MixedPrecisionStep
    wl = W.resnet18()  # inf_every = 100
    kw = wl.step_kwargs()
    ctx = MixedPrecisionStep(wl.numels, **kw)
    specs = [{"numel": n, "grad_dtype": GDT[wl.grad_dtype], "quant": QK[wl.quant]} for n in wl.numels]
    hy = wl.hyper
    sk = {k: kw[k] for k in ("initial_scale", "growth_factor", "backoff_factor", "growth_interval", "min_scale",
                             "max_scale")}
    model = oracle.Model(specs, OPT[wl.optimizer], hy["learning_rate"], beta1=hy["beta1"], beta2=hy["beta2"],
                         epsilon=hy["epsilon"], weight_decay=hy["weight_decay"], scaler_kwargs=sk)
    for i, m in enumerate(wl.master(0)):
        ctx.set_master(i, m)
        model.master[i][:] = m
    qlist = [wl.quant] * len(wl.numels)
    t, skipped, scales = 1, [], []
    for s in range(1, 1001):
        grads = wl.grads(s)
        for i, g in enumerate(grads):
            ctx.set_grad(i, g)
        r = ctx.step(t)
        ro = model.step(grads, t)
        assert r["skipped"] == ro.skipped and r["scale_next"] == ro.scale_next, s
        assert r["step_count"] == ro.step_count == s and r["overflow_count"] == ro.overflow_count, s
        if r["skipped"]:
            skipped.append(s)
            scales.append(r["scale_next"])
        else:
            t += 1
        if s % 100 == 0:
            compare_state(ctx, model, wl.numels, qlist, wl.optimizer)
    assert skipped == list(range(100, 1001, 100))
    assert scales == [65536.0 * 0.5 ** k for k in range(1, 11)]
    ctx.close()
