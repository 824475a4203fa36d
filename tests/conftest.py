import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def weights():
    """Seeded synthetic Flow weights (seed 0, N(0, 0.02)), all 330 tensors."""
    from oracle import flow_oracle as fo
    return fo.synth_weights(seed=0, std=0.02)


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def rel_max(a, b):
    """max|a-b| / max|b| -- the reference's stage metric (tests/verify_flow.py:57-66)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
