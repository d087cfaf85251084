import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and libsc_b200.so")


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("test marked gpu needs a CUDA device (run with -m 'not gpu' on CPU-only hosts)")
    from shardcompute_b200 import _lib

    _lib.load()
    return torch.device("cuda:0")


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
