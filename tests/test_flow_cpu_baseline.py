"""The multithreaded CPU restatement timed as the CPU baseline
(oracle/flow_cpu.py) computes what the pinned numpy oracle computes: one DiT
forward with key-padding and block-causal masks, and a CFG Euler solve
against the reference's own golden vectors."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import golden, rel_max  # noqa: E402
from oracle import flow_oracle as fo  # noqa: E402

TOL = 1e-4   # two float32 evaluation orders of the same network


@pytest.fixture(scope="module")
def cpu(weights):
    from oracle.flow_cpu import FlowCPU
    return FlowCPU(weights)


@pytest.mark.parametrize("chunk", [0, 50])
def test_forward_matches_oracle(cpu, weights, chunk):
    g = golden("dit_chunk.npz" if chunk else "dit_padded.npz")
    L = [int(n) for n in g["lengths"]]
    T = g["x"].shape[-1]
    mask = fo.block_causal_mask(L, T, chunk) if chunk else fo.key_padding_mask(L, T)
    t = np.full(len(L), float(g["t"]), np.float32)
    ref = fo.dit_forward(weights, g["x"], g["mu"], t, g["spks"], g["cond"], mask)
    got = cpu.dit_forward(*(torch.from_numpy(np.ascontiguousarray(a)) for a in (g["x"], g["mu"], t, g["spks"],
                                                                               g["cond"])),
                          torch.from_numpy(mask)).numpy()
    for b, n in enumerate(L):
        assert rel_max(got[b, :, :n], ref[b, :, :n]) < TOL
    if not chunk:
        for b, n in enumerate(L):
            assert rel_max(got[b, :, :n], g["dphi"][b, :, :n]) < 1e-3


def test_solve_matches_golden(cpu):
    g = golden("dit_padded.npz")
    L = [int(n) for n in g["lengths"]]
    T = g["x"].shape[-1]
    mask = torch.from_numpy(fo.key_padding_mask(L, T))
    x = cpu.solve_euler(*(torch.from_numpy(np.ascontiguousarray(g[k])) for k in ("x", "mu", "spks", "cond")),
                        mask).numpy()
    for b, n in enumerate(L):
        assert np.abs(x[b, :, :n] - g["solve"][b, :, :n]).max() < 1e-3
