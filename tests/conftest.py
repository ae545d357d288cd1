"""Shared test fixtures.  GPU tests carry @pytest.mark.gpu and run only on a
B200 (`pytest -m gpu`); everything else runs on a CPU-only machine."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "mlx_quantized.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    """MLX 0.32.3 golden vectors of the reference (tests/golden/make_golden.py)."""
    with np.load(GOLDEN) as d:
        return {k: d[k] for k in d.files}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o
