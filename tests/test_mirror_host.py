"""The Python mirror's host-side logic against the reference's own
assertions, without a GPU: GradientScaler's scalar state machine (the
golden scaler cases, tests/odyssey/training/test_mixed_precision.mojo:29-165)
and PrecisionConfig's modes, dtypes and counters
(tests/odyssey/training/test_precision_config.mojo:65-312)."""
import pytest

import odyssey_b200 as ody


def _apply(s, ops):
    for op in ops:
        (s.step if op == "step" else s.backoff)()


def test_scaler_golden_cases(golden):
    for case in golden["scaler_cases"]["cases"]:
        if "unscale" in case:
            continue  # element work: covered on the GPU
        s = ody.GradientScaler(**case["init"])
        _apply(s, case.get("ops", []))
        exp = case["expect"]
        assert s.scale == exp["scale"], case["name"]
        for k in ("growth_factor", "backoff_factor", "growth_interval"):
            if k in exp:
                assert getattr(s, k) == exp[k], case["name"]
        if "num_steps" in exp:
            assert s.get_num_steps() == exp["num_steps"], case["name"]
        if "then" in case:
            _apply(s, case["then"]["ops"])
            assert s.scale == case["then"]["expect"]["scale"], case["name"]


@pytest.mark.parametrize("name,mode,compute,scaler", [
    ("fp32", "FP32", "float32", False), ("fp16", "FP16", "float16", True),
    ("bf16", "BF16", "bfloat16", True), ("fp8", "FP8", "float16", True)])
def test_precision_config_modes(name, mode, compute, scaler):
    c = ody.PrecisionConfig.from_string(name)
    assert c.mode == getattr(ody.PrecisionMode, mode)
    assert c.compute_dtype == compute and c.storage_dtype == compute
    assert c.master_dtype == "float32"
    assert c.use_gradient_scaler == scaler
    assert c.needs_master_weights() == (name != "fp32")
    if scaler:
        assert c.get_scale() == 65536.0


def test_precision_config_invalid():
    with pytest.raises(ody.OdysseyError, match="Unknown precision: fp64. Use fp32, fp16, bf16, or fp8."):
        ody.PrecisionConfig.from_string("fp64")


def test_precision_config_step_tracking():
    c = ody.PrecisionConfig.fp16()
    assert c.get_step_count() == 0 and c.get_overflow_count() == 0
    c.step(grads_valid=True)
    c.step(grads_valid=True)
    assert c.get_step_count() == 2
    c.step(grads_valid=False)
    assert c.get_overflow_count() == 1 and c.get_step_count() == 3
    assert c.get_scale() == 32768.0  # the backoff halved the scale
