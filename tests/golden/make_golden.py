"""Regenerate the golden fixtures in this folder from the reference project.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/Odyssey

It (1) runs the reference's own numpy/torch parity generators
``tests/odyssey/training/optimizers/parity_refs/{sgd,adam,adamw,lion,rmsprop}_parity_reference.py``
and (2) reads the values the reference's Mojo tests transcribed from them
(``test_{sgd,adam,adamw,lion,rmsprop}.mojo`` ``test_parity_with_reference``), checks that
both agree, and writes ``optimizer_parity.json``.  The scaler and clip cases
(``scaler_cases.json``, ``clip_cases.json``) are the assertions of
``tests/odyssey/training/test_mixed_precision.mojo``,
``tests/odyssey/training/test_gradient_clipping.mojo`` and
``tests/odyssey/core/test_gradient_clipping_simd.mojo`` written as data.

Nothing at test time reads the reference; the tests read only the JSON here.
"""
import json
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OPT_DIR = "tests/odyssey/training/optimizers"


def _run_ref(root, name):
    path = os.path.join(root, OPT_DIR, "parity_refs", f"{name}_parity_reference.py")
    out = subprocess.run([sys.executable, path], check=True, capture_output=True, text=True).stdout
    return json.loads(out[out.index("{"):])


def _mojo_lists(root, name):
    """Values appended to rp/rm/rv (expected) in test_parity_with_reference."""
    src = open(os.path.join(root, OPT_DIR, f"test_{name}.mojo")).read()
    body = src[src.index("def test_parity_with_reference"):]
    body = body[: body.index("print(\"test_parity_with_reference PASSED\")")]
    lists = {}
    for var, val in re.findall(r"\b(r[a-z]+)\.append\(([-0-9.e+]+)\)", body):
        lists.setdefault(var, []).append(float(val))
    call = re.search(rf"{name}_step\(([^)]*)\)", body).group(1)
    line = src[: src.index("def test_parity_with_reference")].count("\n") + 1
    return lists, call, line


def optimizer_parity(root):
    out = {}
    for name in ("sgd", "adam", "adamw", "lion", "rmsprop"):
        ref = _run_ref(root, name)
        lists, call, line = _mojo_lists(root, name)
        new_p = ref["new_params"]
        assert max(abs(a - b) for a, b in zip(new_p, lists["rp"])) < 1e-12, name
        case = {
            "source": f"{OPT_DIR}/test_{name}.mojo:{line} and {OPT_DIR}/parity_refs/{name}_parity_reference.py",
            "mojo_call": f"{name}_step({call})",
            "tolerance": 1e-9,
            "params": ref["params_in"] if "params_in" in ref else ref.get("params"),
            "grad": ref["grad"],
            "new_params": new_p,
        }
        if name == "lion":
            case.update(lr=ref["lr"], beta1=ref["beta1"], beta2=ref["beta2"], weight_decay=ref["weight_decay"],
                        m=ref["momentum_in"], new_m=ref["new_momentum"])
            assert max(abs(a - b) for a, b in zip(ref["new_momentum"], lists["rm"])) < 1e-12
        elif name == "rmsprop":
            case.update(lr=ref["lr"], alpha=ref["alpha"], epsilon=ref["epsilon"], weight_decay=ref["weight_decay"],
                        t=1, square_avg=ref["square_avg_in"], new_square_avg=ref["new_square_avg"],
                        generator=ref["source"])
            assert max(abs(a - b) for a, b in zip(ref["new_square_avg"], lists["rsq"])) < 1e-12
        elif name == "sgd":
            case.update(lr=ref["lr"], momentum=ref["momentum"], weight_decay=ref["weight_decay"],
                        velocity=ref.get("velocity_in", ref.get("velocity")),
                        new_velocity=ref["new_velocity"])
            assert max(abs(a - b) for a, b in zip(ref["new_velocity"], lists["rv"])) < 1e-12
        else:
            case.update(lr=ref["lr"], beta1=ref["beta1"], beta2=ref["beta2"], epsilon=ref["epsilon"],
                        weight_decay=ref["weight_decay"], t=ref["t"], m=ref["m_in"], v=ref["v_in"],
                        new_m=ref["new_m"], new_v=ref["new_v"])
            assert max(abs(a - b) for a, b in zip(ref["new_m"], lists["rm"])) < 1e-12
            assert max(abs(a - b) for a, b in zip(ref["new_v"], lists["rv"])) < 1e-12
        out[name] = case
    return out


SCALER_CASES = {
    "source": "tests/odyssey/training/test_mixed_precision.mojo:29-165",
    "cases": [
        {"name": "defaults", "init": {}, "ops": [],
         "expect": {"scale": 65536.0, "growth_factor": 2.0, "backoff_factor": 0.5,
                    "growth_interval": 2000, "num_steps": 0}},
        {"name": "unscale_2048_by_1024", "init": {"initial_scale": 1024.0},
         "unscale": {"value": 2048.0, "expect": 2.0, "tol": 1e-5}},
        {"name": "growth_at_interval", "init": {"initial_scale": 1024.0, "growth_factor": 2.0,
                                                 "growth_interval": 100},
         "ops": ["step"] * 99, "expect": {"scale": 1024.0},
         "then": {"ops": ["step"], "expect": {"scale": 2048.0}}},
        {"name": "backoff_halves", "init": {"initial_scale": 1024.0, "backoff_factor": 0.5},
         "ops": ["backoff"], "expect": {"scale": 512.0}},
        {"name": "backoff_respects_min", "init": {"initial_scale": 1024.0, "min_scale": 512.0,
                                                   "max_scale": 2048.0, "backoff_factor": 0.5},
         "ops": ["backoff"], "expect": {"scale": 512.0},
         "then": {"ops": ["backoff"], "expect": {"scale": 512.0}}},
        {"name": "growth_caps_at_max", "init": {"initial_scale": 1536.0, "min_scale": 512.0,
                                                 "max_scale": 2048.0, "growth_factor": 2.0,
                                                 "growth_interval": 1},
         "ops": ["step"], "expect": {"scale": 2048.0}},
    ],
}

CLIP_CASES = {
    "source": ("tests/odyssey/training/test_mixed_precision.mojo:316-342; "
               "tests/odyssey/training/test_gradient_clipping.mojo:44-124,262-366; "
               "tests/odyssey/core/test_gradient_clipping_simd.mojo:77-115"),
    "global_norm": [
        {"name": "ones100_twos50_noclip", "tensors": [[1.0, 100], [2.0, 50]], "max_norm": 20.0,
         "expect_norm": 17.320508075688775, "atol": 1e-5, "expect_first": 1.0, "atol_value": 1e-6},
        {"name": "ones100_twos50_clip10", "tensors": [[1.0, 100], [2.0, 50]], "max_norm": 10.0,
         "expect_norm": 17.320508075688775, "atol": 1e-5,
         "expect_first": 10.0 / 17.320508075688775, "atol_value": 1e-5, "expect_new_norm": 10.0,
         "atol_new_norm": 1e-4},
        {"name": "zeros", "tensors": [[0.0, 100]], "max_norm": 1.0, "expect_norm": 0.0, "atol": 1e-6},
        {"name": "ones7", "tensors": [[1.0, 7]], "max_norm": 100.0, "expect_norm": 2.6457513110645907, "atol": 1e-5},
        {"name": "threes13", "tensors": [[3.0, 13]], "max_norm": 100.0, "expect_norm": 10.816653826391969, "atol": 1e-5},
        {"name": "ones33", "tensors": [[1.0, 33]], "max_norm": 100.0, "expect_norm": 5.744562646538029, "atol": 1e-5},
        {"name": "five1", "tensors": [[5.0, 1]], "max_norm": 100.0, "expect_norm": 5.0, "atol": 1e-5},
        {"name": "twos10000_clip10", "tensors": [[2.0, 10000]], "max_norm": 10.0, "expect_norm": 200.0,
         "atol": 1e-3, "expect_new_norm": 10.0, "atol_new_norm": 1e-3},
    ],
    "by_norm": [
        {"name": "345", "values": [3.0, 4.0, 0.0], "max_norm": 1.0, "expect": [0.6, 0.8, 0.0], "atol": 1e-5},
    ],
}


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ODYSSEY_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout>")
    with open(os.path.join(HERE, "optimizer_parity.json"), "w") as f:
        json.dump(optimizer_parity(root), f, indent=1)
    with open(os.path.join(HERE, "scaler_cases.json"), "w") as f:
        json.dump(SCALER_CASES, f, indent=1)
    with open(os.path.join(HERE, "clip_cases.json"), "w") as f:
        json.dump(CLIP_CASES, f, indent=1)
    print("wrote optimizer_parity.json, scaler_cases.json, clip_cases.json")


if __name__ == "__main__":
    main()
