import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "kernel-deltanet_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib():
    """libkdn.so with its signatures (loading needs no GPU)."""
    from kdn_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def rel_err(a, b):
    """max over rows of ||a - b|| / ||b|| (rows = last axis)."""
    import numpy as np

    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    num = np.linalg.norm((a - b).reshape(-1, a.shape[-1]), axis=-1)
    den = np.linalg.norm(b.reshape(-1, b.shape[-1]), axis=-1)
    return float(np.max(num / np.maximum(den, 1e-30)))


def fro_rel(a, b):
    import numpy as np

    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
