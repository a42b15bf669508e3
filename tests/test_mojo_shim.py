"""The reference-side Mojo binding (odyssey_b200/mojo/odyssey_mp.mojo) checked
as text against include/odyssey_mp.h, since no Mojo toolchain exists here:
every get_function[fn (...) -> R]("ody_*") signature has the header's
argument count and types under the binding's C -> Mojo type map, every name
of the update-path boundary is bound, the raw-struct offsets the binding
writes match the C structs, and the reference names it must stand in for
are defined."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "odyssey_b200", "mojo", "odyssey_mp.mojo")
HEADER = os.path.join(ROOT, "include", "odyssey_mp.h")

C_TO_MOJO = {"int32_t": "Int32", "int64_t": "Int64", "uint64_t": "UInt64", "size_t": "UInt64",
             "float": "Float32", "double": "Float64", "int": "Int32", "void": "None"}


def mojo_type(ctype):
    ctype = ctype.strip()
    if "*" in ctype:
        return "OpaquePointer"
    ctype = ctype.replace("const ", "").strip()
    return C_TO_MOJO[ctype]


def header_decls():
    text = re.sub(r"/\*.*?\*/", " ", open(HEADER).read(), flags=re.S)
    decls = {}
    for ret, name, args in re.findall(r"(int64_t|int|void|const char\s*\*)\s*(ody_\w+)\s*\(([^;]*?)\)\s*;", text,
                                      flags=re.S):
        args = " ".join(args.split())
        params = [] if args in ("", "void") else [a.strip() for a in args.split(",")]
        types = []
        for p in params:
            # drop the parameter name: the last identifier, keeping any '*'
            m = re.match(r"(.*?)(\w+)$", p)
            types.append(mojo_type(m.group(1) if m and m.group(1).strip() else p))
        decls[name] = (types, mojo_type(ret))
    return decls


def shim_bindings():
    text = open(SHIM).read()
    sig = r"get_function\[\s*fn\s*\(([^\]]*?)\)\s*->\s*(\w+)\s*\]"
    found = []
    for args, ret, name in re.findall(sig + r"\(\s*\"(ody_\w+)\"\s*\)", text, flags=re.S):
        found.append((name, [a.strip() for a in args.split(",") if a.strip()], ret))
    # helpers that take the entry point's name as an argument
    helpers = {h: re.search(r"def " + h + r"\(.*?" + sig + r"\(name\)", text, flags=re.S)
               for h in ("_quantize", "_dequantize")}
    for h, m in helpers.items():
        assert m, h
        args = [a.strip() for a in m.group(1).split(",") if a.strip()]
        for name in re.findall(h + r"\(\s*\"(ody_\w+)\"", text):
            found.append((name, args, m.group(2)))
    return text, found


REQUIRED = {
    # GradientScaler / PrecisionConfig / free functions of mixed_precision.mojo
    "ody_unscale", "ody_check_finite", "ody_to_fp32", "ody_quantize", "ody_global_norm_clip",
    # optimizers
    "ody_sgd_step", "ody_adam_step", "ody_adamw_step",
    # AnyTensor.to_* / from_*
    "ody_quant_fp8_e4m3", "ody_quant_fp8_e5m2", "ody_quant_mxfp4", "ody_quant_nvfp4",
    "ody_dequant_fp8_e4m3", "ody_dequant_fp8_e5m2", "ody_dequant_mxfp4", "ody_dequant_nvfp4",
    # MixedPrecisionStep
    "ody_config_default", "ody_ctx_create", "ody_ctx_add_tensor", "ody_ctx_finalize", "ody_upload", "ody_step",
    "ody_get_quant", "ody_quant_bytes", "ody_ctx_destroy",
    # errors
    "ody_last_error",
}


def test_every_binding_matches_the_header():
    decls = header_decls()
    assert len(decls) > 50
    _, found = shim_bindings()
    assert found
    for name, args, ret in found:
        assert name in decls, f"{name} is not declared in include/odyssey_mp.h"
        want_args, want_ret = decls[name]
        assert args == want_args, f"{name}: binding {args} != header {want_args}"
        assert ret == want_ret, f"{name}: binding returns {ret}, header {want_ret}"


def test_boundary_names_are_bound():
    _, found = shim_bindings()
    bound = {n for n, _, _ in found}
    assert REQUIRED <= bound, sorted(REQUIRED - bound)


def test_reference_names_defined():
    text, _ = shim_bindings()
    for name in ("struct GradientScaler", "def unscale_gradients", "def step(mut self)", "def backoff",
                 "def convert_to_fp32_master", "def update_model_from_master", "def check_gradients_finite",
                 "def clip_gradients_by_norm", "def clip_gradients_by_global_norm", "def sgd_step",
                 "def adam_step", "def adamw_step", "def init_sgd_state", "def init_adam_state",
                 "def init_adamw_state", "def check_gradients", "def step(mut self, grads_valid: Bool)",
                 "def clip_gradients", "struct MixedPrecisionStep"):
        assert name in text, name
    for fmt in ("fp8", "bf8", "mxfp4", "nvfp4"):
        assert f"def to_{fmt}(" in text and f"def from_{fmt}(" in text, fmt


def test_struct_offsets_match_the_c_layout():
    L = pytest.importorskip("odyssey_b200._lib")
    import ctypes as C
    text, _ = shim_bindings()
    consts = {k: int(v) for k, v in re.findall(r"comptime (\w+) = (\d+)\n", text)}
    assert consts["CONFIG_BYTES"] == C.sizeof(L.Config)
    assert consts["RESULT_BYTES"] == C.sizeof(L.StepResult)
    cfg = {"CFG_OPTIMIZER": "optimizer", "CFG_DEVICE": "device", "CFG_LR": "learning_rate",
           "CFG_MOMENTUM": "momentum", "CFG_BETA1": "beta1", "CFG_BETA2": "beta2", "CFG_EPSILON": "epsilon",
           "CFG_WEIGHT_DECAY": "weight_decay", "CFG_USE_SCALER": "use_gradient_scaler",
           "CFG_INITIAL_SCALE": "initial_scale", "CFG_GROWTH_FACTOR": "growth_factor",
           "CFG_BACKOFF_FACTOR": "backoff_factor", "CFG_GROWTH_INTERVAL": "growth_interval",
           "CFG_MIN_SCALE": "min_scale", "CFG_MAX_SCALE": "max_scale", "CFG_CLIP_ENABLED": "clip_enabled",
           "CFG_MAX_NORM": "max_norm"}
    for k, f in cfg.items():
        assert consts[k] == getattr(L.Config, f).offset, k
    res = {"RES_SKIPPED": "skipped", "RES_CLIPPED": "clipped", "RES_GRAD_NORM": "grad_norm",
           "RES_SCALE_NEXT": "scale_next"}
    for k, f in res.items():
        assert consts[k] == getattr(L.StepResult, f).offset, k


def test_constants_match_the_header():
    text, _ = shim_bindings()
    hdr = open(HEADER).read()
    hv = {k: int(v) for k, v in re.findall(r"#define (ODY_\w+) \(?(-?\d+)\)?", hdr)}
    for k, v in re.findall(r"comptime (ODY_\w+): Int32 = (-?\d+)", text):
        assert hv[k] == int(v), k
