"""GPU parity of the re-quantisation kernels against the oracle: bit-exact
codes, block scales and per-tensor scales for every kind, on seeded inputs,
ragged sizes and the special values the reference's tests use."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

KINDS = [1, 2, 3, 4, 5, 6, 7, 8, 9]  # FP16 .. NVFP4_TENSOR, MXFP4 by the OCP MX rule


@pytest.fixture(scope="module")
def ody():
    import odyssey_b200 as o
    o.lib()
    return o


def _specials():
    return np.float32([0.0, -0.0, np.nan, np.inf, -np.inf, 1e-45, -1e-45, 1e-38, 6.0, -6.0, 0.5, 1.25, 1.75, 2.5,
                       3.5, 5.0, 448.0, 500.0, 65504.0, 1e30, -1e-7, 3e-8])


def _mixed(n, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    x *= np.float32(10.0) ** rng.integers(-6, 3, n).astype(np.float32)
    return x


def _gpu_quant(ody, kind, x, src_dtype=0):
    out = np.zeros(ody._lib.quant_bytes(kind, x.size), np.uint8)
    ts = C.c_float(0)
    ody._lib.check(ody.lib().ody_quantize(kind, x.ctypes.data, src_dtype, x.size, out.ctypes.data, C.byref(ts)))
    return out, ts.value


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("n", [1, 15, 16, 17, 31, 33, 2047, 2048, 2049, 100003])
def test_quantize_bit_exact_ragged(ody, oracle, kind, n):
    x = _mixed(n, n + kind)
    if kind in (1, 2, 3, 4, 6, 7):  # finite specials for the plain kinds
        sp = _specials()
        k = min(n, sp.size)
        x[:k] = sp[:k]
    if kind in (5, 8):
        x = np.nan_to_num(x, nan=0.0, posinf=7.0, neginf=-7.0)
    got, ts = _gpu_quant(ody, kind, x)
    want, wts = oracle.quantize(kind, x)
    np.testing.assert_array_equal(got, want)
    assert np.float32(ts) == np.float32(wts)


@pytest.mark.parametrize("kind", [6, 7, 8])
def test_quantize_bf16_source(ody, oracle, kind):
    from odyssey_b200.workloads import bf16_bits_to_f32, f32_to_bf16_bits
    h = f32_to_bf16_bits(_mixed(5000, 3) * np.float32(0.02))
    got, ts = _gpu_quant(ody, kind, h, src_dtype=2)
    want, wts = oracle.quantize(kind, bf16_bits_to_f32(h))
    np.testing.assert_array_equal(got, want)
    assert np.float32(ts) == np.float32(wts)


def test_e4m3_cast_sweep(ody, oracle):
    """Hardware cvt.rn.satfinite e4m3 (the NVFP4 block-scale byte) against the
    oracle's software RNE on every 97th float32 bit pattern of [0, 480]."""
    bits = np.arange(0, 0x43F00000, 97, dtype=np.uint32)
    x = bits.view(np.float32)
    x = np.concatenate([x, -x])
    got, _ = _gpu_quant(ody, 3, x)
    want, _ = oracle.quantize(3, x)
    np.testing.assert_array_equal(got, want)


def test_e5m2_f16_bf16_cast_sweep(ody, oracle):
    bits = np.arange(0x30000000, 0x47800000, 131, dtype=np.uint32)
    x = np.concatenate([bits.view(np.float32), -bits.view(np.float32)])
    for kind in (1, 2, 4):
        got, _ = _gpu_quant(ody, kind, x)
        want, _ = oracle.quantize(kind, x)
        np.testing.assert_array_equal(got, want, err_msg=f"kind {kind}")


@pytest.mark.parametrize("kind", [6, 7, 8])
def test_fp4_threshold_tables_every_scale(ody, oracle, kind):
    """For every block scale the table-driven encode equals the reference's
    division ladder: blocks whose amax selects each E8M0/E4M3 scale, filled
    with values straddling every threshold."""
    B = 32 if kind == 6 else 16
    rng = np.random.default_rng(7)
    blocks = []
    exps = range(-40, 40) if kind == 6 else np.linspace(-11, 9, 400)
    for e in exps:
        amax = np.float32(6.0 * 2.0 ** e)
        vals = amax * rng.uniform(-1, 1, B).astype(np.float32)
        t = np.float32([0.5, 1.25, 1.75, 2.5, 3.5, 5.0])
        sc = amax / np.float32(6.0)
        k = min(B - 1, 6)
        vals[1:k + 1] = t[:k] * sc * np.float32(1 + 1e-7 * rng.standard_normal())
        vals[0] = amax
        blocks.append(vals)
    x = np.concatenate(blocks).astype(np.float32)
    got, ts = _gpu_quant(ody, kind, x)
    want, wts = oracle.quantize(kind, x)
    np.testing.assert_array_equal(got, want)


def _ulp_sweep(c, k):
    """float32 values k ulps either side of each c (same sign), c included."""
    b = np.asarray(c, np.float32).view(np.int32).astype(np.int64)
    out = (b[:, None] + np.arange(-k, k + 1)[None, :]).ravel()
    out = out[(out > 0) & (out < 0x7F800000)]
    return out.astype(np.int32).view(np.float32)


def _boundary_blocks(B, scales, mult, rng, tiny=True):
    """Blocks of B elements: element 0 = 6 * scale * mult (selects the block
    scale), the rest sweep the ladder break points T * scale * mult and the
    smallest quotients, +-8 ulps, both signs."""
    T = np.float32([0.5, 1.25, 1.75, 2.5, 3.5, 5.0])
    blocks = []
    for sc in scales:
        sc = np.float32(sc)
        parts = [_ulp_sweep(T * sc * np.float32(mult), 8)]
        if tiny:
            parts.append(_ulp_sweep(np.float32([2.0 ** -149, 2.0 ** -148, 1e-40]) * sc, 3))
        pts = np.concatenate(parts)
        pts = pts * np.where(rng.random(pts.size) < 0.5, np.float32(-1), np.float32(1))
        head = np.float32(6.0) * sc * np.float32(mult)
        for i in range(0, pts.size, B - 1):
            blk = np.zeros(B, np.float32)
            chunk = pts[i:i + B - 1]
            blk[1:1 + chunk.size] = chunk
            blk[0] = head
            blocks.append(blk)
    return np.concatenate(blocks)


@pytest.mark.parametrize("kind", [6, 7, 8])
def test_fp4_encode_break_points_every_scale(ody, oracle, kind):
    """The one-thread-per-block encoder (exact quotient + top-16-bit ladder)
    against the oracle's IEEE division at every ladder break point +-8 ulps,
    for every block scale the format reaches: all E4M3 codes (NVFP4), E8M0
    exponents 2^-120..2^120 (MXFP4), and for the per-tensor-scaled NVFP4
    several tensor scales (the tensor amax set by one extra element)."""
    rng = np.random.default_rng(11)
    if kind == 6:
        scales = 2.0 ** np.arange(-120, 121, 3, dtype=np.float64)
        x = _boundary_blocks(32, scales, 1.0, rng)
        got, _ = _gpu_quant(ody, kind, x)
        want, _ = oracle.quantize(kind, x)
        np.testing.assert_array_equal(got, want)
        return
    e4m3 = oracle.e4m3_to_f32(np.arange(1, 127, dtype=np.uint8))
    mults = [1.0] if kind == 7 else [1.0, 3.7e-5, 1e-3, 2.5e7]
    # per-tensor: with subnormal-range elements (the sign decided by the
    # threshold t0) and without (every nonzero quotient normal: the sign
    # comes with the quotient)
    for mult, tiny in [(m, t) for m in mults for t in ((True,) if kind == 7 else (True, False))]:
        x = _boundary_blocks(16, e4m3, mult, rng, tiny)
        if kind == 8:
            # the tensor's amax (one more block) sets s_t = amax / 2688, so
            # that q = x / s_t puts block scales on every E4M3 code
            tail = np.zeros(16, np.float32)
            tail[0] = np.float32(2688.0 * mult)
            x = np.concatenate([x, tail])
        got, ts = _gpu_quant(ody, kind, x)
        want, wts = oracle.quantize(kind, x)
        np.testing.assert_array_equal(got, want, err_msg=f"mult {mult} tiny {tiny}")
        assert np.float32(ts) == np.float32(wts)


def test_mxfp4_ocp_rounding_every_scale(ody, oracle):
    """MXFP4 by the OCP MX rule (hardware E2M1 conversion, round to nearest
    even, saturating) against the oracle at every rounding midpoint of the
    E2M1 grid +-4 ulps, shared exponents 2^-130..2^125, both signs, signed
    zeros, and blocks whose amax sits exactly on a power of two."""
    rng = np.random.default_rng(5)
    mids = np.float32([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.5, 1.0, 4.0])
    blocks = []
    for X in range(-130, 126, 3):
        sc = np.float32(2.0 ** X)
        pts = _ulp_sweep(mids * sc, 4) if sc * 0.25 > 1e-37 else np.float32(mids * sc)
        pts = pts * np.where(rng.random(pts.size) < 0.5, np.float32(-1), np.float32(1))
        for i in range(0, pts.size, 31):
            blk = np.zeros(32, np.float32)
            chunk = pts[i:i + 31]
            blk[1:1 + chunk.size] = chunk
            blk[0] = np.float32(4.0) * sc  # amax exactly 2^(X+2): shared exponent X
            if i % 2:
                blk[31] = np.float32(-0.0)
            blocks.append(blk)
    x = np.concatenate(blocks)
    got, _ = _gpu_quant(ody, 9, x)
    want, _ = oracle.quantize(9, x)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("kind", KINDS)
def test_dequantize_bit_exact(ody, oracle, kind):
    x = np.nan_to_num(_mixed(4099, kind), nan=0.0, posinf=1.0, neginf=-1.0)
    q, ts = oracle.quantize(kind, x)
    out = np.zeros(x.size, np.float32)
    ody._lib.check(ody.lib().ody_dequantize(kind, q.ctypes.data, x.size, ts, out.ctypes.data))
    want = oracle.dequantize(kind, q, x.size, ts)
    np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))


def test_every_code_byte_decodes(ody, oracle):
    """Decode of all 256 byte values for each FP4 / FP8 kind."""
    for kind in (3, 4, 6, 7):
        if kind in (6, 7):
            B = 17 if kind == 6 else 9
            nb = 256
            q = np.zeros(nb * B, np.uint8)
            for b in range(nb):
                q[b * B: b * B + B - 1] = b
                q[b * B + B - 1] = (b * 37) % (256 if kind == 6 else 127)
            n = nb * (32 if kind == 6 else 16)
        else:
            q = np.arange(256, dtype=np.uint8)
            n = 256
        out = np.zeros(n, np.float32)
        ody._lib.check(ody.lib().ody_dequantize(kind, q.ctypes.data, n, 1.0, out.ctypes.data))
        want = oracle.dequantize(kind, q, n, 1.0)
        np.testing.assert_array_equal(np.isnan(out), np.isnan(want))
        m = ~np.isnan(want)
        np.testing.assert_array_equal(out[m].view(np.uint32), want[m].view(np.uint32))


def test_python_mirror_api(ody, oracle):
    x = _mixed(1000, 11)
    q = ody.to_mxfp4(x)
    want, _ = oracle.quantize(6, x)
    np.testing.assert_array_equal(q.data, want)
    np.testing.assert_array_equal(ody.from_mxfp4(q), oracle.dequantize(6, want, x.size))
    with pytest.raises(ody.OdysseyError, match="multiple of 17"):
        ody.from_mxfp4(np.zeros(18, np.uint8))
    q = ody.to_nvfp4_tensor_scaled(x)
    w, s = oracle.quantize(8, x)
    np.testing.assert_array_equal(q.data, w)
    assert q.tensor_scale == s


def test_device_pointers_via_torch(ody, oracle):
    torch = pytest.importorskip("torch")
    x = _mixed(70000, 5)
    xd = torch.from_numpy(x).cuda()
    q = ody.to_nvfp4(xd)
    assert q.data.is_cuda
    want, _ = oracle.quantize(7, x)
    np.testing.assert_array_equal(q.data.cpu().numpy(), want)
    d = ody.from_nvfp4(q.data)
    np.testing.assert_array_equal(d.cpu().numpy()[: x.size], oracle.dequantize(7, want, x.size))


@pytest.mark.parametrize("kind", [6, 7, 8])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_fp4_device_source_alignments(ody, oracle, kind, offset):
    """Device sources that start 0, 4 or 12 bytes past a 16-byte boundary
    (the staged path needs 16-byte alignment; the others take the direct
    one), float32 and bfloat16, ragged length: both paths bit-exact."""
    torch = pytest.importorskip("torch")
    x = _mixed(50001, 9 + offset)
    base = torch.from_numpy(np.concatenate([np.zeros(offset, np.float32), x])).cuda()
    got = np.zeros(ody._lib.quant_bytes(kind, x.size), np.uint8)
    ts = C.c_float(0)
    ody._lib.check(ody.lib().ody_quantize(kind, base[offset:].data_ptr(), 0, x.size, got.ctypes.data, C.byref(ts)))
    want, wts = oracle.quantize(kind, x)
    np.testing.assert_array_equal(got, want)
    assert np.float32(ts.value) == np.float32(wts)
    from odyssey_b200.workloads import f32_to_bf16_bits, bf16_bits_to_f32
    hb = f32_to_bf16_bits(x)
    bb = torch.from_numpy(np.concatenate([np.zeros(offset, np.uint16), hb]).view(np.int16)).cuda()
    ody._lib.check(ody.lib().ody_quantize(kind, bb[offset:].data_ptr(), 2, x.size, got.ctypes.data, C.byref(ts)))
    want, wts = oracle.quantize(kind, bf16_bits_to_f32(hb))
    np.testing.assert_array_equal(got, want)


def test_config2_full_size_mxfp4(ody, oracle):
    """Config 2 at full size (4096^2): bit-exact codes and round trip."""
    from odyssey_b200.workloads import mxfp4_tensor
    x = mxfp4_tensor(0)
    got, _ = _gpu_quant(ody, 6, x)
    want, _ = oracle.quantize(6, x)
    np.testing.assert_array_equal(got, want)
    out = np.zeros(x.size, np.float32)
    ody._lib.check(ody.lib().ody_dequantize(6, got.ctypes.data, x.size, 1.0, out.ctypes.data))
    np.testing.assert_array_equal(out, oracle.dequantize(6, want, x.size))


def test_config3_full_size_nvfp4_bf16(ody, oracle):
    """Config 3 at full size (8192^2 BF16) with the per-tensor scale and
    without it (pure reference to_nvfp4)."""
    from odyssey_b200.workloads import bf16_bits_to_f32, nvfp4_tensor_bf16
    h = nvfp4_tensor_bf16(0)
    xf = bf16_bits_to_f32(h)
    for kind in (8, 7):
        got, ts = _gpu_quant(ody, kind, h, src_dtype=2)
        want, wts = oracle.quantize(kind, xf)
        np.testing.assert_array_equal(got, want)
        assert np.float32(ts) == np.float32(wts)


def test_exact_division_shortcut(ody):
    """The requant's reciprocal + one-remainder-correction division equals
    IEEE division bit for bit, over random scales spanning the float32 range
    and the per-tensor scales of real weights."""
    import ctypes as C
    torch = pytest.importorskip("torch")
    g = torch.Generator(device="cuda").manual_seed(0)
    n = 1 << 24
    for lo, hi in ((-30.0, 30.0), (-120.0, 120.0), (-14.0, -6.0)):
        x = (torch.randn(n, device="cuda", generator=g) * torch.exp2(torch.empty(n, device="cuda").uniform_(
            lo, hi, generator=g))).float()
        s = torch.exp2(torch.empty(n, device="cuda").uniform_(lo, hi, generator=g)).float()
        s = s * (1 + torch.rand(n, device="cuda", generator=g))
        fast, ieee = torch.empty_like(x), torch.empty_like(x)
        f = ody.lib().odyx_selftest_divide
        f.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]
        assert f(x.data_ptr(), s.data_ptr(), n, fast.data_ptr(), ieee.data_ptr()) == 0
        bad = (fast.view(torch.int32) != ieee.view(torch.int32)).nonzero().flatten()
        if bad.numel():
            i = bad[:5].tolist()
            pytest.fail(f"{bad.numel()} mismatches, e.g. x={x[i].tolist()} s={s[i].tolist()} "
                        f"fast={fast[i].tolist()} ieee={ieee[i].tolist()}")


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
def test_fp4_singles_bit_exact(ody, oracle, fmt):
    """MXFP4/NVFP4.from_float32, from_float32_stochastic and to_float32 per
    value (mxfp4.mojo:303-491, nvfp4.mojo:290-481) against the oracle: codes
    and scale bytes bit for bit over magnitudes from subnormal to the float
    maximum, zeros of both signs, NaN and Inf, and seeds over the full 64
    bits (the LCG uses their low 32)."""
    rng = np.random.default_rng(11)
    n = 20000
    x = (np.exp2(rng.uniform(-149, 127.9, n)) * rng.choice([-1.0, 1.0], n)).astype(np.float32)
    x[:2000] = (rng.standard_normal(2000) * 3).astype(np.float32)
    x[2000:2010] = [0.0, -0.0, np.nan, np.inf, -np.inf, 1.25, -1.25, 6.0, 0.5, 3.4e38]
    seeds = rng.integers(0, 2**63, n, dtype=np.int64).astype(np.uint64) * np.uint64(2) + np.uint64(1)
    kind = ody.MXFP4.kind if fmt == "mxfp4" else ody.NVFP4.kind
    cls = ody.MXFP4 if fmt == "mxfp4" else ody.NVFP4
    for sd in (None, seeds):
        v, s = cls.from_float32(x) if sd is None else cls.from_float32_stochastic(x, sd)
        ov, os_ = oracle.fp4_single_encode(kind, x, sd)
        np.testing.assert_array_equal(v, ov)
        np.testing.assert_array_equal(s, os_)
        d = cls.to_float32(v, s)
        od = oracle.fp4_single_decode(kind, v, s)
        np.testing.assert_array_equal(d.view(np.uint32), od.view(np.uint32))


def test_fp4_single_stochastic_is_unbiased(ody):
    """from_float32_stochastic: 1.25 between 1.0 and 1.5 rounds up about half
    the time over many seeds (mxfp4.mojo:361-366)."""
    n = 100000
    seeds = np.arange(n, dtype=np.uint64) * np.uint64(2654435761)
    v, s = ody.MXFP4.from_float32_stochastic(np.full(n, 1.25, np.float32), seeds)
    d = ody.MXFP4.to_float32(v, s)
    assert set(np.unique(d).tolist()) <= {1.0, 1.5}
    assert abs(d.mean() - 1.25) < 0.01


@pytest.mark.parametrize("fmt,kind", [("mxfp4", 6), ("nvfp4", 7), ("fp8_e4m3", 3), ("fp8_e5m2", 4), ("fp16", 1),
                                      ("bf16", 2)])
def test_per_format_entry_points(ody, oracle, fmt, kind):
    """ody_quant_<fmt> / ody_dequant_<fmt> equal the generic calls and the oracle."""
    x = _mixed(5000, 21)
    lib = ody.lib()
    out = np.zeros(ody._lib.quant_bytes(kind, x.size), np.uint8)
    ody._lib.check(getattr(lib, f"ody_quant_{fmt}")(x.ctypes.data, 0, x.size, out.ctypes.data))
    ref, _ = _gpu_quant(ody, kind, x)
    np.testing.assert_array_equal(out, ref)
    ora = np.zeros(oracle.quant_bytes(kind, x.size), np.uint8)
    oracle.lib().ora_quantize(kind, x.ctypes.data, x.size, ora.ctypes.data)
    np.testing.assert_array_equal(out, ora[: out.size])
    back = np.zeros(x.size, np.float32)
    ody._lib.check(getattr(lib, f"ody_dequant_{fmt}")(out.ctypes.data, x.size, back.ctypes.data))
    oback = np.zeros(x.size, np.float32)
    oracle.lib().ora_dequantize(kind, ora.ctypes.data, x.size, 1.0, oback.ctypes.data)
    np.testing.assert_array_equal(back.view(np.uint32), oback.view(np.uint32))


@pytest.mark.parametrize("kind", KINDS)
def test_quantize_on_stream_matches(ody, kind):
    """ody_quantize_on_stream / ody_dequantize_on_stream (device memory,
    stream-ordered) equal the synchronous calls."""
    import torch
    x = _mixed(70001, 31)
    ref, ts_ref = _gpu_quant(ody, kind, x)
    dx = torch.from_numpy(x).cuda()
    out = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
    ts = torch.zeros(1, dtype=torch.float32, device="cuda")
    scratch = torch.zeros(2, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    ody._lib.check(ody.lib().ody_quantize_on_stream(kind, dx.data_ptr(), 0, x.size, out.data_ptr(), ts.data_ptr(),
                                                     scratch.data_ptr(), st))
    back = torch.zeros(x.size, dtype=torch.float32, device="cuda")
    ody._lib.check(ody.lib().ody_dequantize_on_stream(kind, out.data_ptr(), x.size, ts.data_ptr(), back.data_ptr(),
                                                       st))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    assert ts.item() == np.float32(ts_ref) or kind not in (5, 8)
    hb = np.zeros(x.size, np.float32)
    ody._lib.check(ody.lib().ody_dequantize(kind, ref.ctypes.data, x.size, ts_ref, hb.ctypes.data))
    np.testing.assert_array_equal(back.cpu().numpy().view(np.uint32), hb.view(np.uint32))
    with pytest.raises(ody.OdysseyError, match="device memory only"):
        ody._lib.check(ody.lib().ody_quantize_on_stream(kind, x.ctypes.data, 0, x.size, out.data_ptr(),
                                                         ts.data_ptr(), scratch.data_ptr(), st))


def test_to_family_float64_and_float16_sources(ody, oracle):
    """to_fp8/to_mxfp4 accept float64 (rounded to float32, the reference's
    .cast[DType.float32]) and float16 (exact upcast) sources."""
    x64 = np.random.default_rng(4).standard_normal(5000) * 3.0
    x32 = x64.astype(np.float32)
    np.testing.assert_array_equal(ody.to_fp8(x64).data, ody.to_fp8(x32).data)
    np.testing.assert_array_equal(ody.to_mxfp4(x64).data, oracle.quantize(6, x32)[0])
    x16 = x32.astype(np.float16)
    np.testing.assert_array_equal(ody.to_bf8(x16).data, oracle.quantize(4, x16.astype(np.float32))[0])
