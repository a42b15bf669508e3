"""bench.py's bookkeeping on CPU: the algorithmic bytes per unit of every
workload (the scope table's figures), the workload configs, and the
reference arm's JSON line."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("name,quant,expect", [("flat1b", "nvfp4_tensor", 26.5625), ("lenet", "fp16", 20.0),
                                               ("resnet18", "fp8_tensor", 27.0)])
def test_alg_bytes_per_param(name, quant, expect):
    wl = bench.make_workload(name, 64)
    assert bench.alg_bytes_per_param(wl, quant) == expect


def test_quant_workload_bytes():
    assert bench.QUANT_WORKLOADS["mxfp4"]["bytes_per_elem"] == 4 + 17 / 32
    assert bench.QUANT_WORKLOADS["nvfp4"]["bytes_per_elem"] == 2 + 2 + 9 / 16


def test_workload_sizes():
    assert bench.make_workload("flat1b", 64).total == 1073741824
    assert bench.make_workload("lenet", 64).total == 61706
    assert bench.make_workload("resnet18", 64).total == 11173962


def test_reference_arm_line():
    """--impl reference prints one JSON line with the contract's keys (the
    oracle timed on the host; a short sample)."""
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "lenet",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    line = json.loads(p.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
