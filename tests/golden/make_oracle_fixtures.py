#!/usr/bin/env python3
"""Oracle outputs for the benchmarked shapes, too slow to recompute per test run.

The numpy oracle (``oracle/flow_oracle.py``, itself pinned to vectors the
reference's own ``tests/flow_reference.py`` produced) takes minutes for a full
10-step decode at these sizes, so the results are computed once here and the
GPU tests compare against the stored arrays.  Inputs are NOT stored: both this
script and the tests rebuild them from the seeds with ``parity_inputs`` below
(numpy's PCG64 ``Generator.standard_normal`` stream).

  oracle_cfg2_T1000.npz  BASELINE config 2: one T=1000 utterance, 10-step
                         cosine CFM Euler with CFG 2, full attention.
                         mel [80, 1000] (the final x of every frame).
  oracle_cfg4_ctx500.npz BASELINE config 4 at its worst context: 8 streams of
                         500 context + 50 chunk + 6 look-ahead = 556 frames,
                         block-causal chunk mask (chunk 50), 10-step CFG.
                         mel [8, 80, 556].

Weights: ``fo.synth_weights(seed=0, std=0.02)`` (the same seeded tensors the
GPU tests write to a flow.gguf).  Run once (about 8 minutes on 8 cores):
    python tests/golden/make_oracle_fixtures.py
"""

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import flow_oracle as fo  # noqa: E402

CFG2 = {"seed": 2, "lengths": [1000], "chunk": 0}
CFG4 = {"seed": 4, "lengths": [556] * 8, "chunk": 50}


def parity_inputs(lengths, seed):
    """Per utterance [80, T] mu / cond / noise and spks [U, 80]: N(0,1) mu,
    spks and noise, cond N(0,1) over the first 20% of frames (the benchmark's
    input distribution).  Returns lists of arrays and the spks matrix."""
    rng = np.random.default_rng(seed)
    mus, conds, noises = [], [], []
    for L in lengths:
        mus.append(rng.standard_normal((80, L), dtype=np.float32))
        noises.append(rng.standard_normal((80, L), dtype=np.float32))
        c = np.zeros((80, L), np.float32)
        p = int(0.2 * L)
        c[:, :p] = rng.standard_normal((80, p), dtype=np.float32)
        conds.append(c)
    spks = rng.standard_normal((len(lengths), 80), dtype=np.float32)
    return mus, conds, spks, noises


def solve(W, case):
    L = case["lengths"]
    T = max(L)
    assert all(n == T for n in L), "fixtures use equal lengths (no padding in the oracle batch)"
    mus, conds, spks, noises = parity_inputs(L, case["seed"])
    mask = fo.block_causal_mask(L, T, case["chunk"]) if case["chunk"] else None
    return fo.solve_euler(W, np.stack(noises), np.stack(mus), spks, np.stack(conds), mask)


def main():
    W = fo.synth_weights(seed=0, std=0.02)
    for name, case in (("oracle_cfg2_T1000.npz", CFG2), ("oracle_cfg4_ctx500.npz", CFG4)):
        t0 = time.time()
        mel = solve(W, case)
        out = {"mel": mel[0] if len(case["lengths"]) == 1 else mel, "seed": np.int64(case["seed"]),
               "lengths": np.asarray(case["lengths"], np.int32), "chunk": np.int64(case["chunk"])}
        np.savez_compressed(os.path.join(HERE, name), **out)
        print(f"{name}: {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main()
