import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def _load(name):
    z = np.load(os.path.join(GOLDEN, name))
    cases = {}
    for key in z.files:
        case, arr = key.split("/", 1)
        cases.setdefault(case, {})[arr] = z[key]
    return cases


@pytest.fixture(scope="session")
def golden_op():
    return _load("golden_op.npz")


@pytest.fixture(scope="session")
def golden_layer():
    return _load("golden_layer.npz")
