"""GPU parity of the single-op entry points (unscale, finite check, global-
norm clip, SGD / Adam / AdamW / Lion / RMSprop / Adagrad) against the oracle
and the reference's golden vectors."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ody():
    import odyssey_b200 as o
    o.lib()
    return o


def _rand(n, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


@pytest.mark.parametrize("name", ["sgd", "adam", "adamw"])
def test_golden_vectors_f32(ody, golden, name):
    """The reference's float64 golden vectors, through the float32 kernels:
    within float32 rounding of the 1e-9 float64 answers."""
    c = golden["optimizer_parity"][name]
    f = lambda k: np.array(c[k], np.float32)  # noqa: E731
    if name == "sgd":
        p, v = ody.sgd_step(f("params"), f("grad"), f("velocity"), c["lr"], c["momentum"], c["weight_decay"])
        np.testing.assert_allclose(v, c["new_velocity"], rtol=2e-6, atol=1e-8)
    else:
        fn = ody.adam_step if name == "adam" else ody.adamw_step
        p, m, v = fn(f("params"), f("grad"), f("m"), f("v"), c["t"], c["lr"], c["beta1"], c["beta2"],
                     c["epsilon"], c["weight_decay"])
        np.testing.assert_allclose(m, c["new_m"], rtol=2e-6, atol=1e-9)
        np.testing.assert_allclose(v, c["new_v"], rtol=2e-6, atol=1e-12)
    np.testing.assert_allclose(p, c["new_params"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("n", [1, 7, 1000, 65537])
@pytest.mark.parametrize("wd", [0.0, 0.01])
def test_optimizers_bit_exact(ody, oracle, n, wd):
    p, g, m = _rand(n, 1, 0.05), _rand(n, 2, 1e-3), _rand(n, 3, 1e-3)
    v = np.abs(_rand(n, 4, 1e-6))
    a = ody.sgd_step(p, g, m, 0.01, 0.9, wd)
    b = oracle.sgd_step(p, g, m, 0.01, 0.9, wd)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x.view(np.uint32), y.view(np.uint32))
    for t in (1, 7, 1000):
        a = ody.adam_step(p, g, m, v, t, 1e-3, 0.9, 0.999, 1e-8, wd)
        b = oracle.adam_step(p, g, m, v, t, 1e-3, 0.9, 0.999, 1e-8, wd)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x.view(np.uint32), y.view(np.uint32))
        a = ody.adamw_step(p, g, m, v, t, 1e-3, 0.9, 0.999, 1e-8, wd)
        b = oracle.adamw_step(p, g, m, v, t, 1e-3, 0.9, 0.999, 1e-8, wd)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("n", [1, 7, 1000, 65537])
@pytest.mark.parametrize("wd", [0.0, 0.01])
def test_lion_rmsprop_adagrad_bit_exact(ody, oracle, n, wd):
    """lion.mojo / rmsprop.mojo / adagrad.mojo through the CUDA single ops,
    bit for bit against the oracle's float32 restatement; zeros in the
    gradient and momentum exercise Lion's sign(0) = 0."""
    p, g, m = _rand(n, 1, 0.05), _rand(n, 2, 1e-3), _rand(n, 3, 1e-3)
    g[::5] = 0.0
    m[::5] = 0.0
    sq = np.abs(_rand(n, 4, 1e-6))
    same = lambda a, b: [np.testing.assert_array_equal(x.view(np.uint32), y.view(np.uint32))  # noqa: E731
                         for x, y in zip(a, b)]
    same(ody.lion_step(p, g, m, 1e-4, 0.9, 0.99, wd), oracle.lion_step(p, g, m, 1e-4, 0.9, 0.99, wd))
    same(ody.adagrad_step(p, g, sq, 1e-2, 1e-10, wd), oracle.adagrad_step(p, g, sq, 1e-2, 1e-10, wd))
    a = ody.rmsprop_step(p, g, sq, 1, 1e-2, 0.99, 1e-8, wd)
    b = oracle.rmsprop_step(p, g, sq, 1e-2, 0.99, 1e-8, wd)
    same(a[:2], b[:2])
    buf = _rand(n, 5, 1e-2)
    a = ody.rmsprop_step(p, g, sq, 3, 1e-2, 0.9, 1e-8, wd, momentum=0.9, buf=buf)
    b = oracle.rmsprop_step(p, g, sq, 1e-2, 0.9, 1e-8, wd, momentum=0.9, buf=buf)
    same(a, b)


@pytest.mark.parametrize("name", ["lion", "rmsprop"])
def test_lion_rmsprop_golden_f32(ody, golden, name):
    """The reference's float64 golden vectors (test_lion.mojo,
    test_rmsprop.mojo) through the float32 kernels."""
    c = golden["optimizer_parity"][name]
    f = lambda k: np.array(c[k], np.float32)  # noqa: E731
    if name == "lion":
        p, m = ody.lion_step(f("params"), f("grad"), f("m"), c["lr"], c["beta1"], c["beta2"], c["weight_decay"])
        np.testing.assert_allclose(m, c["new_m"], rtol=2e-6, atol=1e-9)
    else:
        p, sq, _ = ody.rmsprop_step(f("params"), f("grad"), f("square_avg"), 1, c["lr"], c["alpha"],
                                    c["epsilon"], c["weight_decay"])
        np.testing.assert_allclose(sq, c["new_square_avg"], rtol=2e-6, atol=1e-12)
    np.testing.assert_allclose(p, c["new_params"], rtol=2e-6, atol=1e-7)


def test_optimizer_errors(ody):
    z = np.zeros(4, np.float32)
    with pytest.raises(ody.OdysseyError, match="Timestep t must be positive"):
        ody.adamw_step(z, z, z, z, 0, 1e-3)
    with pytest.raises(ody.OdysseyError, match="Velocity buffer required"):
        ody.sgd_step(z, z, None, 0.1, momentum=0.9)
    with pytest.raises(ody.OdysseyError, match="same shape"):
        ody.sgd_step(z, np.zeros(5, np.float32), z, 0.1)
    with pytest.raises(ody.OdysseyError, match="lion_step: params and momentum must have the same shape"):
        ody.lion_step(z, z, np.zeros(5, np.float32), 1e-4)
    with pytest.raises(ody.OdysseyError, match="square_avg must be initialized"):
        ody.rmsprop_step(z, z, np.zeros(0, np.float32), 1, 1e-2)
    with pytest.raises(ody.OdysseyError, match="Timestep t must be positive"):
        ody.rmsprop_step(z, z, z, 0, 1e-2)
    with pytest.raises(ody.OdysseyError, match="accumulator must be initialized"):
        ody.adagrad_step(z, z, np.zeros(0, np.float32), 1e-2)


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_unscale_and_check(ody, oracle, dtype):
    from odyssey_b200.workloads import f32_to_bf16_bits
    x = _rand(10001, 9, 1024.0)
    x[5] = np.float32(70000.0)
    code = {"float32": 0, "float16": 1, "bfloat16": 2}[dtype]
    g = x if dtype == "float32" else (x.astype(np.float16) if dtype == "float16" else f32_to_bf16_bits(x))
    s = ody.GradientScaler(initial_scale=1024.0)
    out = s.unscale_gradients(g, dtype=dtype if dtype == "bfloat16" else None)
    want = oracle.unscale(g, 1024.0, dtype=code)
    np.testing.assert_array_equal(np.asarray(out).view(np.uint8), want.view(np.uint8))
    ok = ody.check_gradients_finite(g, dtype=dtype if dtype == "bfloat16" else None)
    assert ok == (oracle.count_nonfinite(g, dtype=code) == 0)
    # NaN / +-Inf detection (test_mixed_precision.mojo:209-286)
    for bad in ("nan", "inf", "-inf"):
        gb = g.copy()
        gb[3] = {"float32": np.float32(bad), "float16": np.float16(bad),
                 "bfloat16": f32_to_bf16_bits(np.float32([bad]))[0]}[dtype]
        assert not ody.check_gradients_finite(gb, dtype=dtype if dtype == "bfloat16" else None)


def test_unscale_fp16_scale_overflow(ody, oracle):
    """full(F64(65536), float16) is +inf: g/inf = 0 and inf/inf = NaN, as the reference."""
    g = np.float16([1.0, -2.0, np.inf, 0.0])
    s = ody.GradientScaler()
    out = s.unscale_gradients(g)
    want = oracle.unscale(g, 65536.0)
    np.testing.assert_array_equal(out.view(np.uint16)[:2], want.view(np.uint16)[:2])
    assert np.isnan(out[2]) and np.isnan(want[2])


def test_global_norm_clip_cases(ody, golden):
    for case in golden["clip_cases"]["global_norm"]:
        grads = [np.full(n, v, np.float32) for v, n in case["tensors"]]
        norm = ody.clip_gradients_by_global_norm(grads, case["max_norm"])
        assert abs(norm - case["expect_norm"]) <= case["atol"], case["name"]
        if "expect_first" in case:
            assert abs(grads[0][0] - case["expect_first"]) <= case["atol_value"], case["name"]
        if "expect_new_norm" in case:
            assert abs(ody.compute_gradient_norm_list(grads) - case["expect_new_norm"]) <= case["atol_new_norm"]
    c = golden["clip_cases"]["by_norm"][0]
    out = ody.clip_gradients_by_norm(np.float32(c["values"]), c["max_norm"])
    np.testing.assert_allclose(out, c["expect"], atol=c["atol"])
    with pytest.raises(ody.OdysseyError, match="max_norm must be positive"):
        ody.clip_gradients_by_global_norm([np.zeros(3, np.float32)], 0.0)


def test_global_norm_clip_vs_oracle(ody, oracle):
    grads = [_rand(n, n, 3.0) for n in (1, 100, 70001, 1 << 20)]
    a = [g.copy() for g in grads]
    b = [g.copy() for g in grads]
    na = ody.clip_gradients_by_global_norm(a, 1.0)
    nb = oracle.global_norm_clip(b, 1.0)
    assert na == nb
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def _cast_cases(half_bits, seed):
    """float32 inputs for a cast to a 16-bit format: random magnitudes across
    the format's range (subnormals and overflow included), exact midpoints
    between neighbouring codes (ties, both parities), the values one float32
    ulp either side of those ties, and the specials."""
    rng = np.random.default_rng(seed)
    up = ((lambda h: h.astype(np.float32)) if half_bits == "f16"
          else (lambda h: (h.astype(np.uint32) << 16).view(np.float32)))
    codes = rng.integers(0, 0x7C00 if half_bits == "f16" else 0x7F80, 20000).astype(np.uint16)
    lo = up(codes.view(np.float16) if half_bits == "f16" else codes)
    hi = up((codes + 1).view(np.float16) if half_bits == "f16" else codes + 1)
    mid = ((lo.astype(np.float64) + hi.astype(np.float64)) / 2).astype(np.float32)  # exact in float32
    near = np.concatenate([np.nextafter(mid, np.float32(np.inf)), np.nextafter(mid, np.float32(0))])
    rnd = (rng.standard_normal(20000) * np.exp2(rng.uniform(-30, 20, 20000))).astype(np.float32)
    spec = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 65504.0, 65520.0, 65519.996, 6e-8, 3e-8, 2.9e-8,
                     np.float32(3.4e38)], np.float32)
    x = np.concatenate([lo, mid, near, rnd, spec])
    sign = np.where(rng.random(x.size) < 0.5, np.float32(-1.0), np.float32(1.0))
    return np.concatenate([x, x * sign]).astype(np.float32)


def test_master_conversions(ody, oracle):
    """update_model_from_master (mixed_precision.mojo:299-354) rounds to
    FP16 / BF16 to nearest even: bit-exact against the oracle on random,
    tie, near-tie, subnormal, overflow and special inputs; and
    convert_to_fp32_master (:240-296) is the exact upcast of every FP16 and
    BF16 bit pattern."""
    for fmt, seed in (("f16", 1), ("bf16", 2)):
        x = _cast_cases(fmt, seed)
        if fmt == "f16":
            model = np.zeros(x.size, np.float16)
            ody.update_model_from_master(model, x)
            got = model.view(np.uint16)
            want = oracle.f32_to_f16_bits(x)
        else:
            model = np.zeros(x.size, np.uint16)
            ody.update_model_from_master(model, x, dtype="bfloat16")
            got = model
            want = oracle.f32_to_bf16_bits(x)
        nan = np.isnan(x)
        np.testing.assert_array_equal(got[~nan], want[~nan], err_msg=fmt)
        assert np.all(np.isnan(oracle.upcast(got[nan], 1 if fmt == "f16" else 2)))
    every = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    m16 = ody.convert_to_fp32_master(every.view(np.float16))
    want16 = oracle.upcast(every.view(np.float16))
    nan16 = np.isnan(want16)  # the 2,046 NaN codes: NaN out (the payload is not part of the contract)
    np.testing.assert_array_equal(m16.view(np.uint32)[~nan16], want16.view(np.uint32)[~nan16])
    assert np.all(np.isnan(m16[nan16]))
    mb = ody.convert_to_fp32_master(every, dtype="bfloat16")
    np.testing.assert_array_equal(mb.view(np.uint32), (every.astype(np.uint32) << 16))
    p = np.full(100, 1.0, np.float16)
    with pytest.raises(ody.OdysseyError, match="sizes must match"):
        ody.update_model_from_master(p, np.zeros(3, np.float32))


def test_single_ops_refuse_another_gpus_memory(ody):
    """A device buffer of a GPU other than the current one is refused with
    ODY_ERR_ARG before any launch."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.cuda.set_device(0)
    g = torch.ones(64, dtype=torch.float32, device="cuda:1")
    with pytest.raises(ody.OdysseyError, match="another GPU") as ei:
        ody.GradientScaler().unscale_gradients(g)
    assert ei.value.code == -1


@pytest.mark.parametrize("mode", [0, 1])
def test_clip_variants(ody, oracle, mode):
    """clip_grad_global_norm_ (mode 0) and clip_global_norm (mode 1): the
    norm within float64 summation-order rounding of the reference's, the
    clipped values bit-exact given that norm, and the reference's example
    (ones(100), ones(50), max 5 -> norm sqrt(150))."""
    fn = ody.clip_grad_global_norm_ if mode == 0 else ody.clip_global_norm
    g = [_rand(1000, 1, 3.0), _rand(37, 2, 0.5), _rand(70001, 3, 0.01)]
    orig = [x.copy() for x in g]
    norm = fn(g, 2.0)
    if mode == 0:
        ref = math.sqrt(sum(oracle.sumsq_f32(x) for x in orig))
    else:
        ref = math.sqrt(sum(float(np.sum(x.astype(np.float64) ** 2)) for x in orig))
    assert abs(norm - ref) <= 1e-12 * ref
    for a, o in zip(g, orig):
        want = o * np.float32(2.0 / norm) if mode == 0 else (o.astype(np.float64) * (2.0 / norm)).astype(np.float32)
        np.testing.assert_array_equal(a.view(np.uint32), want.astype(np.float32).view(np.uint32))
    # below the bound: untouched
    h = [_rand(100, 4, 1e-3)]
    h0 = h[0].copy()
    fn(h, 100.0)
    np.testing.assert_array_equal(h[0], h0)
    a, b = np.ones(100, np.float32), np.ones(50, np.float32)
    n = fn([a, b], 5.0)
    assert n == pytest.approx(math.sqrt(150.0), rel=1e-12)
    np.testing.assert_allclose(a, 5.0 / math.sqrt(150.0), rtol=1e-6)
