"""CPU checks of the C ABI: libodyssey_mp.so loads, exports every symbol
include/odyssey_mp.h declares, and its host-only logic (defaults, byte
counts, shard plan, argument validation) behaves without a GPU."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def L():
    from odyssey_b200 import _lib
    from odyssey_b200.build import build
    build()
    _lib.lib()
    return _lib


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "odyssey_mp.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ody_\w+)\s*\(", src)))


def test_header_symbols_exported(L):
    names = declared_symbols()
    assert len(names) >= 34
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (ody_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert hasattr(L.lib(), n)
    # the Python binding covers exactly the header
    assert sorted(L.EXPORTED) == names


def test_build_targets_sm100a_only():
    from odyssey_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    for flag in ("-fmad=false", "-ftz=false", "-prec-div=true", "-prec-sqrt=true"):
        assert flag in build.NVFLAGS
    assert "--use_fast_math" not in build.NVFLAGS


def test_defaults_match_reference(L):
    c = L.default_config()
    # GradientScaler() defaults (mixed_precision.mojo:96-122)
    assert (c.initial_scale, c.growth_factor, c.backoff_factor, c.growth_interval, c.min_scale, c.max_scale) == \
        (65536.0, 2.0, 0.5, 2000, 1.0, 65536.0)
    assert (c.beta1, c.beta2, c.epsilon) == (0.9, 0.999, 1e-8)
    assert L.lib().ody_abi_version() == 1


def test_quant_bytes(L):
    q = L.quant_bytes
    assert q(L.Q_MXFP4, 32) == 17 and q(L.Q_MXFP4, 33) == 34 and q(L.Q_MXFP4, 4096 * 4096) == 8912896
    assert q(L.Q_NVFP4, 8192 * 8192) == 37748736 and q(L.Q_NVFP4_TENSOR, 1) == 9
    assert q(L.Q_FP16, 5) == 10 and q(L.Q_FP8_E4M3, 5) == 5 and q(L.Q_NONE, 5) == 0 and q(99, 5) == -1


def test_plan_shards(L):
    from odyssey_b200 import plan_shards
    # config 5: 64 equal tensors -> 64/N whole tensors per rank
    for n in (1, 2, 4, 8):
        own = plan_shards([4096 * 4096] * 64, n)
        assert [own.count(r) for r in range(n)] == [64 // n] * n
        assert own == sorted(own)
    # ResNet-18: contiguous, every tensor owned once, balanced within the largest tensor
    from odyssey_b200.workloads import RESNET18_SHAPES, numels
    ns = numels(RESNET18_SHAPES)
    for n in (2, 4, 8):
        own = plan_shards(ns, n)
        assert own == sorted(own) and len(own) == len(ns)
        loads = [sum(x for x, r in zip(ns, own) if r == k) for k in range(n)]
        assert max(loads) - sum(ns) / n <= max(ns)


def test_create_and_validation_without_gpu(L):
    ctx = C.c_void_p()
    cfg = L.default_config()
    cfg.optimizer = 7
    assert L.lib().ody_ctx_create(C.byref(ctx), C.byref(cfg)) == L.ERR_ARG
    assert "unknown optimizer" in L.last_error()
    cfg = L.default_config()
    cfg.clip_enabled, cfg.max_norm = 1, 0.0
    assert L.lib().ody_ctx_create(C.byref(ctx), C.byref(cfg)) == L.ERR_ARG
    assert L.last_error().startswith("max_norm must be positive")
    cfg = L.default_config()
    assert L.lib().ody_ctx_create(C.byref(ctx), C.byref(cfg)) == L.OK
    assert L.lib().ody_ctx_add_tensor(ctx, 0, L.BF16, L.Q_NVFP4, None) == L.ERR_SHAPE
    assert L.lib().ody_ctx_add_tensor(ctx, 10, L.BF16, 42, None) == L.ERR_ARG
    idx = C.c_int32(-1)
    assert L.lib().ody_ctx_add_tensor(ctx, 10, L.BF16, L.Q_NVFP4, C.byref(idx)) == L.OK and idx.value == 0
    assert L.lib().ody_ctx_add_tensor(ctx, 10, L.F16, L.Q_NVFP4, None) == L.ERR_DTYPE
    assert L.lib().ody_step(ctx, 1, None) == L.ERR_STATE
    assert "not finalized" in L.last_error(ctx)
    L.lib().ody_ctx_destroy(ctx)


def test_stateless_errors_without_gpu(L):
    z = np.zeros(4, np.float32)
    assert L.lib().ody_unscale(z.ctypes.data, L.F32, 0, 2.0, z.ctypes.data) == L.ERR_SHAPE
    assert L.last_error() == "Cannot unscale empty gradient tensor"
    assert L.lib().ody_unscale(z.ctypes.data, L.F32, 4, 0.0, z.ctypes.data) == L.ERR_ARG
    assert L.last_error() == "Cannot unscale with zero scale factor"
    assert L.lib().ody_adamw_step(z.ctypes.data, z.ctypes.data, z.ctypes.data, z.ctypes.data, 4, 0, 1e-3, 0.9,
                                  0.999, 1e-8, 0.0, z.ctypes.data, z.ctypes.data, z.ctypes.data) == L.ERR_ARG
    assert L.last_error() == "Timestep t must be positive (starts at 1)"


def test_no_cpu_fallback(L):
    """Without a GPU the compute entry points fail loudly (status CUDA)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    z = np.ones(4, np.float32)
    rc = L.lib().ody_unscale(z.ctypes.data, L.F32, 4, 2.0, z.ctypes.data)
    assert rc == L.ERR_CUDA
    from odyssey_b200 import OdysseyError, to_nvfp4
    with pytest.raises(OdysseyError):
        to_nvfp4(z)


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    from odyssey_b200 import _lib
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "absent.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(_lib.OdysseyError, match="missing"):
        _lib.lib()


@pytest.mark.parametrize("compiler", [["gcc", "-std=c11"], ["g++", "-x", "c++", "-std=c++17"]])
def test_c_caller(L, tmp_path, compiler):
    """tests/abi_check.c: the header and library used from plain C (gcc) and
    C++ (g++), host-only entry points and error paths."""
    exe = tmp_path / "abi_check"
    libdir = os.path.dirname(L.LIB_PATH)
    cc = subprocess.run(compiler + ["-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                                    os.path.join(ROOT, "tests", "abi_check.c"), "-o", str(exe), "-L", libdir,
                                    "-l:" + os.path.basename(L.LIB_PATH), f"-Wl,-rpath,{libdir}"],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr


def test_reference_source_checks_of_to_family():
    """AnyTensor.to_fp8/to_bf8/to_mxfp4/to_nvfp4 reject bfloat16 and
    non-float sources with the reference's messages
    (tests/odyssey/tensor/test_fp8_bf8_conversion.mojo:18-116,
    tensor_dtype_conv.mojo:21-36,259-279); checked before any device work."""
    import torch
    from odyssey_b200 import OdysseyError, to_bf8, to_fp8, to_mxfp4, to_nvfp4
    for fn, name in ((to_fp8, "to_fp8()"), (to_bf8, "to_bf8()"), (to_mxfp4, "to_mxfp4()"),
                     (to_nvfp4, "to_nvfp4()")):
        with pytest.raises(OdysseyError, match=re.escape(f"{name} does not support bfloat16: the bfloat16 "
                                                         "conversion path does not correctly round-trip")):
            fn(torch.zeros(2, 3, dtype=torch.bfloat16))
        with pytest.raises(OdysseyError, match="does not support bfloat16"):
            fn(np.zeros(6, np.uint16), dtype="bfloat16")
        with pytest.raises(OdysseyError, match=re.escape(f"{name} requires a floating-point tensor")):
            fn(np.zeros(6, np.int32))


def test_reference_checks_of_from_family():
    """from_fp8/from_bf8/from_mxfp4/from_nvfp4 source checks
    (tensor_dtype_conv.mojo:78-79,227-228,380-385,444-449)."""
    from odyssey_b200 import OdysseyError, from_bf8, from_fp8, from_mxfp4, from_nvfp4
    for fn, what in ((from_fp8, "FP8"), (from_bf8, "BF8"), (from_mxfp4, "MXFP4"), (from_nvfp4, "NVFP4")):
        with pytest.raises(OdysseyError, match=re.escape(f"from_{what.lower()}() requires a uint8 tensor "
                                                         f"({what}-encoded)")):
            fn(np.zeros(18, np.float32))
    with pytest.raises(OdysseyError, match="MXFP4 tensor size must be multiple of 17 bytes"):
        from_mxfp4(np.zeros(18, np.uint8))
    with pytest.raises(OdysseyError, match="NVFP4 tensor size must be multiple of 9 bytes"):
        from_nvfp4(np.zeros(10, np.uint8))


def test_chunk_elems_validation(L):
    import ctypes as C
    cfg = L.default_config()
    ctx = C.c_void_p()
    for bad in (-2048, 1000, 131072):
        cfg.chunk_elems = bad
        assert L.lib().ody_ctx_create(C.byref(ctx), C.byref(cfg)) == L.ERR_ARG
    cfg.chunk_elems = 4096
    assert L.lib().ody_ctx_create(C.byref(ctx), C.byref(cfg)) == 0
    L.lib().ody_ctx_destroy(ctx)


def test_clip_variants_argument_errors():
    """clip_grad_global_norm_ / clip_global_norm messages
    (numerical_safety.mojo:775-778, optimizer_utils.mojo:326-329), raised
    before any device work."""
    from odyssey_b200 import OdysseyError, clip_global_norm, clip_grad_global_norm_
    with pytest.raises(OdysseyError, match="max_norm must be non-negative, got: -1"):
        clip_grad_global_norm_([np.ones(4, np.float32)], -1.0)
    with pytest.raises(OdysseyError, match="grads list cannot be empty"):
        clip_grad_global_norm_([], 1.0)
    with pytest.raises(OdysseyError, match="tensors list cannot be empty"):
        clip_global_norm([], 1.0)
