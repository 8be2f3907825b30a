"""Shared pytest setup. GPU tests are marked ``gpu`` and run on a B200 box
(``pytest -m gpu``); everything else runs on the CPU (``-m "not gpu"``)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def normwise(x, ref) -> float:
    """max|x - ref| / max|ref|: the parity metric (elementwise relative error
    is fragile near zero, see gemm_selftest's 200x50x300 case)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(x - ref).max() / (den if den > 0 else 1.0))


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name + ".npz"))
    return load


@pytest.fixture(scope="session")
def orc():
    from oracle import orc as o
    o.build()
    return o


@pytest.fixture(scope="session")
def dgx():
    import torch
    import dreamcompiler_b200 as d
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    d.init(0)
    return d
