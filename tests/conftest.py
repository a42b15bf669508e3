import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the libodyssey_mp.so kernels")


@pytest.fixture(scope="session")
def oracle():
    """The C oracle (test infrastructure), built on first use."""
    from oracle import oracle as O
    O.build()
    O.lib()
    return O


@pytest.fixture(scope="session")
def golden():
    import json
    d = os.path.join(ROOT, "tests", "golden")
    return {k: json.load(open(os.path.join(d, f"{k}.json"))) for k in ("optimizer_parity", "scaler_cases",
                                                                       "clip_cases")}
