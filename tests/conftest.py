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


def packed_starts(lengths):
    """Row offsets of packed sequences (each starts on an 8-row boundary, the
    layout of lx_flow_op_attention) and the total packed row count."""
    starts, r = [], 0
    for L in lengths:
        starts.append(r)
        r += (L + 7) // 8 * 8
    return starts, r


def attn_ref_fp64(q, k, v, lengths, starts, chunk):
    """softmax(q k^T / 8 + mask) v per head in float64 over packed [R, 1024]
    rows (full attention, or the block-causal chunk mask when chunk > 0)."""
    from oracle import flow_oracle as fo
    out = np.zeros_like(q)
    for L, s in zip(lengths, starts):
        mask = fo.block_causal_mask([L], L, chunk)[0] if chunk else np.ones((L, L), bool)
        qs, ks, vs = q[s:s + L], k[s:s + L], v[s:s + L]
        for h in range(16):
            sl = slice(64 * h, 64 * h + 64)
            sc = (qs[:, sl] @ ks[:, sl].T) / 8.0
            sc = np.where(mask, sc, -np.inf)
            p = np.exp(sc - sc.max(-1, keepdims=True))
            out[s:s + L, sl] = (p / p.sum(-1, keepdims=True)) @ vs[:, sl]
    return out
