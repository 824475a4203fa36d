"""Parity of the benchmarked kernel instances at the benchmarked shapes.

The projection GEMMs run on the CTA-pair kernel (k_gemm2: QKV with the
rotary / fp16-V epilogue, FF1 with GELU, out and FF2 with the residual-loader
warp) only when a problem has at least two waves of 256 x 256 pair tiles
(roughly >= 3.1k packed rows for QKV, 4.8k for FF1, 9.5k for out / FF2), so
the small parity cases of test_gpu_flow.py run the 1-CTA kernel.  This file
covers the pair kernels and the BASELINE shapes:

  * the small golden / oracle cases again in a subprocess that forces every
    projection onto the pair kernel (LX_FLOW_PAIR_GEMM=2);
  * one estimator forward over the first 8 utterances of the config-3 set
    (6045 frames, 12090 packed rows: every pair kernel in its default
    selection) against the oracle, and against the same utterances run one
    at a time (1-CTA kernels) -- each sequence is independent, so both must
    agree;
  * the config-2 decode (one T=1000 utterance, 10 CFG Euler steps) and 8
    config-4 streams at 500 frames of context (556 frames, chunk 50) against
    oracle results stored by tests/golden/make_oracle_fixtures.py.

Tolerances as in test_gpu_flow.py: per-stage rel-max (max|d| / max|ref|)
within the reference's 1e-2 gate, final mel max-abs <= 2e-2 after 10 steps.
"""

import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import GOLDEN, REPO, golden, rel_l2, rel_max
from oracle import flow_oracle as fo

sys.path.insert(0, GOLDEN)
from make_oracle_fixtures import CFG2, CFG4, parity_inputs  # noqa: E402

pytestmark = pytest.mark.gpu

STAGE_TOL = 1e-2
MEL_ABS_TOL = 2e-2
PATH_TOL = 1e-3   # pair vs 1-CTA kernels on the same inputs (rel-L2 of dphi)


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    from larynx_b200.weights import write_synthetic_gguf
    p = str(tmp_path_factory.mktemp("w") / "flow_synth.gguf")
    write_synthetic_gguf(p, seed=0, std=0.02)
    return p


@pytest.fixture(scope="module")
def dec(gguf_path):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    from larynx_b200 import FlowDecoder
    d = FlowDecoder(0)
    assert d.load(gguf_path), d.last_error
    yield d
    d.close()


def _flat(a):
    return np.concatenate([np.asarray(x, np.float32).reshape(-1) for x in a])


def _split(flat, lengths):
    out, o = [], 0
    for L in lengths:
        out.append(flat[o:o + 80 * L].reshape(80, L))
        o += 80 * L
    return out


def test_small_cases_on_forced_pair_kernels():
    """The golden and oracle cases of test_gpu_flow.py with every projection
    GEMM on the CTA-pair kernel (the switch is read once per process)."""
    tests = ["test_estimator_stages_fixture", "test_estimator_vs_oracle_long", "test_estimator_block_causal",
             "test_decode_padded_batch_golden", "test_infer_fixture", "test_decode_chunked_vs_oracle"]
    env = dict(os.environ, LX_FLOW_PAIR_GEMM="2")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "gpu",
                        os.path.join(REPO, "tests", "test_gpu_flow.py"), "-k", " or ".join(tests)],
                       cwd=REPO, env=env, capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert f"{len(tests)} passed" in r.stdout, r.stdout[-2000:]


def _cfg3_subset():
    """The first 8 utterances of the benchmark's config-3 set (seed 3)."""
    lengths = [int(n) for n in np.random.default_rng(3).integers(100, 1501, 64)[:8]]
    mus, conds, spks, noises = parity_inputs(lengths, seed=33)
    return lengths, mus, conds, spks, noises


def _cfg_rows(lengths, mus, conds, spks, noises):
    """Each utterance as its conditional sequence and its CFG-zeroed sequence
    (mu, cond, spks zeroed) at the same x: the estimator batch of one step."""
    L2, xs, m2, c2, s2 = [], [], [], [], []
    for i, n in enumerate(lengths):
        L2 += [n, n]
        xs += [noises[i], noises[i]]
        m2 += [mus[i], np.zeros_like(mus[i])]
        c2 += [conds[i], np.zeros_like(conds[i])]
        s2 += [spks[i], np.zeros_like(spks[i])]
    return L2, xs, m2, c2, np.stack(s2)


def test_cfg3_scale_estimator_pair_kernels(dec, weights):
    lengths, mus, conds, spks, noises = _cfg3_subset()
    L2, xs, m2, c2, s2 = _cfg_rows(lengths, mus, conds, spks, noises)
    assert 2 * sum(lengths) >= 37 * 256   # out / FF2 pair threshold: 2 waves of 148 SMs / 2
    t = 0.3
    dphi, _ = dec.estimator(L2, _flat(xs), _flat(m2), _flat(c2), s2, t)
    big = _split(dphi, L2)
    assert all(np.isfinite(d).all() for d in big)
    # the same utterances one at a time (<= 2634 rows: 1-CTA kernels throughout)
    for i, n in enumerate(lengths):
        d1, _ = dec.estimator([n, n], _flat(xs[2 * i:2 * i + 2]), _flat(m2[2 * i:2 * i + 2]),
                              _flat(c2[2 * i:2 * i + 2]), s2[2 * i:2 * i + 2], t)
        for j, d in enumerate(_split(d1, [n, n])):
            e = rel_l2(big[2 * i + j], d)
            assert e < PATH_TOL, (i, j, e)
    # the shortest and the longest utterance against the oracle
    for i in (int(np.argmin(lengths)), int(np.argmax(lengths))):
        ref = fo.dit_forward(weights, np.stack(xs[2 * i:2 * i + 2]), np.stack(m2[2 * i:2 * i + 2]),
                             np.full(2, t, np.float32), s2[2 * i:2 * i + 2], np.stack(c2[2 * i:2 * i + 2]))
        for j in range(2):
            assert rel_max(big[2 * i + j], ref[j]) < STAGE_TOL, (i, j)
            assert rel_l2(big[2 * i + j], ref[j]) < STAGE_TOL, (i, j)


def _decode_vs_fixture(dec, case, name):
    g = golden(name)
    L = case["lengths"]
    mus, conds, spks, noises = parity_inputs(L, case["seed"])
    out = dec.decode(L, mus, conds, spks, noise=noises, chunk=case["chunk"])
    ref = g["mel"].reshape(len(L), 80, max(L))
    errs = [float(np.abs(m - ref[u]).max()) for u, m in enumerate(_split(out, L))]
    assert max(errs) < MEL_ABS_TOL, errs
    return errs


def test_cfg2_T1000_decode_vs_oracle(dec):
    """a 20 s utterance, the full 10-step CFG decode."""
    _decode_vs_fixture(dec, CFG2, "oracle_cfg2_T1000.npz")


def test_cfg4_ctx500_streams_vs_oracle(dec):
    """BASELINE config 4 at its worst context: 8 streams x (500 context + 50
    chunk + 6 look-ahead), block-causal chunk mask 50, 10-step CFG decode
    (8896 packed rows: QKV and FF1 on the pair kernel)."""
    _decode_vs_fixture(dec, CFG4, "oracle_cfg4_ctx500.npz")


_ROW_ORDER_CHILD = r"""
import sys
import numpy as np
repo, golden_dir, gguf, out_path = sys.argv[1:5]
sys.path[:0] = [repo, golden_dir]
from larynx_b200 import FlowDecoder
from make_oracle_fixtures import parity_inputs
lengths = [120, 700, 333, 1000, 250, 560]
mus, conds, spks, noises = parity_inputs(lengths, seed=44)
d = FlowDecoder(0)
assert d.load(gguf), d.last_error
np.save(out_path, d.decode(lengths, mus, conds, spks, noise=noises))
d.close()
"""


def test_row_order_is_bit_identical(gguf_path, tmp_path):
    """The decode packs sequences longest first and alternates the row
    direction of AdaLN and the pair GEMMs (for L2 reuse between kernels);
    with LX_FLOW_ROW_ORDER=0 it packs in input order and runs every kernel
    upward.  Each row and tile is computed the same way in either order, so
    the two decodes must agree bit for bit.  Every projection is forced onto
    the pair kernel so that its reversed schedule runs (both switches are read
    once per process, hence the child processes)."""
    outs = {}
    for v in ("0", "1"):
        path = str(tmp_path / f"mel_{v}.npy")
        env = dict(os.environ, LX_FLOW_ROW_ORDER=v, LX_FLOW_PAIR_GEMM="2")
        r = subprocess.run([sys.executable, "-c", _ROW_ORDER_CHILD, REPO, GOLDEN, gguf_path, path],
                           cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        outs[v] = np.load(path)
    assert np.isfinite(outs["1"]).all()
    assert np.array_equal(outs["0"], outs["1"])
