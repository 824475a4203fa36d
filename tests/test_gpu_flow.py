"""End-to-end parity of the CUDA Flow path (through the C ABI) against the
oracle and the reference's golden vectors.

Tolerances (north star): per-stage rel-max (max|d| / max|ref|, the
reference's own stage metric, tests/verify_flow.py:57-66) within the
reference's GREEN gate of 1e-2, and final mel max-abs <= 2e-2 after all 10
Euler steps with bf16 activations / fp32 accumulation and residual stream.
"""

import os

import numpy as np
import pytest

from conftest import golden, rel_l2, rel_max
from oracle import flow_oracle as fo

pytestmark = pytest.mark.gpu

STAGE_TOL = 1e-2     # reference GREEN gate per stage (README.md:187-199)
MEL_ABS_TOL = 2e-2   # final mel max-abs after 10 steps (north star)


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


def test_estimator_stages_fixture(dec, weights):
    """One DiT forward of the reference fixture's step-1 batch ([x; x] rows)."""
    g = golden("flow_fixture.npz")
    T = g["mu"].shape[-1]
    x = g["noise_z"][0]
    mu = g["mu"][0]
    cond = g["cond"][0]
    spk = g["spk"][0]
    xs = [x, x]
    mus = [mu, np.zeros_like(mu)]
    conds = [cond, np.zeros_like(cond)]
    spks = np.stack([spk, np.zeros_like(spk)])
    for blk in (0, 10, 21):
        dphi, cap = dec.estimator([T, T], _flat(xs), _flat(mus), _flat(conds), spks, 0.0, capture_block=blk,
                                  want_input_embed=True, want_norm_out=True)
        got_blk = cap["block"].reshape(2, T, 1024)
        assert rel_max(got_blk, g[f"dit_block{blk}"]) < STAGE_TOL, blk
    assert rel_max(cap["input_embed"].reshape(2, T, 1024), g["dit_input_embed_step1"]) < STAGE_TOL
    assert rel_max(cap["norm_out"].reshape(2, T, 1024), g["dit_norm_out_step1"]) < STAGE_TOL
    d = np.stack(_split(dphi, [T, T]))
    assert rel_max(d, g["dphi_step1"]) < STAGE_TOL


def test_estimator_vs_oracle_long(dec, weights):
    """Random inputs, T = 300 and 129 (several 128-row tiles, ragged tail)."""
    rng = np.random.default_rng(5)
    L = [300, 129]
    xs = [rng.standard_normal((80, n)).astype(np.float32) for n in L]
    mus = [rng.standard_normal((80, n)).astype(np.float32) for n in L]
    conds = [np.where(np.arange(n) < n // 5, rng.standard_normal((80, n)), 0).astype(np.float32) for n in L]
    spks = rng.standard_normal((2, 80)).astype(np.float32)
    dphi, _ = dec.estimator(L, _flat(xs), _flat(mus), _flat(conds), spks, 0.42)
    got = _split(dphi, L)
    for i, n in enumerate(L):
        ref = fo.dit_forward(weights, xs[i][None], mus[i][None], np.array([0.42], np.float32), spks[i:i + 1],
                             conds[i][None])[0]
        assert rel_max(got[i], ref) < STAGE_TOL
        assert rel_l2(got[i], ref) < STAGE_TOL


def test_estimator_block_causal(dec, weights):
    g = golden("dit_chunk.npz")
    L = [int(n) for n in g["lengths"]]
    xs = [g["x"][b, :, :n] for b, n in enumerate(L)]
    mus = [g["mu"][b, :, :n] for b, n in enumerate(L)]
    conds = [g["cond"][b, :, :n] for b, n in enumerate(L)]
    dphi, _ = dec.estimator(L, _flat(xs), _flat(mus), _flat(conds), g["spks"], float(g["t"]), chunk=int(g["chunk"]))
    for b, d in enumerate(_split(dphi, L)):
        assert rel_max(d, g["dphi"][b, :, :L[b]]) < STAGE_TOL


def test_decode_padded_batch_golden(dec):
    """Key-padding batch (lengths 20, 32): 10-step CFG solve vs the golden."""
    g = golden("dit_padded.npz")
    L = [int(n) for n in g["lengths"]]
    out = dec.decode(L, [g["mu"][b, :, :n] for b, n in enumerate(L)], [g["cond"][b, :, :n] for b, n in enumerate(L)],
                     g["spks"], noise=[g["x"][b, :, :n] for b, n in enumerate(L)])
    for b, m in enumerate(_split(out, L)):
        ref = g["solve"][b, :, :L[b]]
        assert np.abs(m - ref).max() < MEL_ABS_TOL


# The stage table of the reference's own verifier (tests/verify_flow.py:37-50):
# (stage, golden key, shape of the capture); plus the 22 blocks.
VERIFY_STAGES = (
    ("spk", "spk", (1, 80)),
    ("token_embed", "token_embed", (1, 12, 80)),
    ("prelookahead", "prelookahead", (1, 12, 80)),
    ("mu", "mu", (1, 80, 24)),
    ("cond", "cond", (1, 80, 24)),
    ("time_embed", "time_embed_step1", (2, 1024)),
    ("input_proj", "dit_input_proj_step1", (2, 24, 1024)),
    ("conv_pos", "dit_conv_pos_step1", (2, 24, 1024)),
    ("input_embed", "dit_input_embed_step1", (2, 24, 1024)),
    ("norm_out", "dit_norm_out_step1", (2, 24, 1024)),
    ("dphi", "dphi_step1", (2, 80, 24)),
)


def test_infer_fixture(dec, weights):
    """Token-level infer (frontend + 10-step decode) on the reference's own
    24-frame validation case: every stage of the reference's FlowDebug,
    checked as its verifier checks it (rel = max|d| / max|ref| within the 1e-2
    gate), against the golden vectors the reference produced; the 22 block
    outputs against the golden where it holds them (blocks 0, 10, 21) and
    against the oracle's step-1 captures for all 22."""
    g = golden("flow_fixture.npz")
    dbg = {}
    mel = dec.infer(g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0], g["spk_embedding"][0],
                    noise_z=g["noise_z"][0], debug=dbg)
    assert mel is not None
    assert mel.shape == g["feat"][0].shape
    assert np.abs(mel - g["feat"][0]).max() < MEL_ABS_TOL
    assert rel_max(mel, g["feat"][0]) < STAGE_TOL
    for stage, key, shape in VERIFY_STAGES:
        got = dbg[stage]
        assert got.size == int(np.prod(shape)), stage
        assert rel_max(got.reshape(shape), g[key]) < STAGE_TOL, stage
    # the frontend runs in fp32 on both sides: much tighter than the gate
    assert rel_max(dbg["spk"], g["spk"][0]) < 1e-5
    assert rel_max(dbg["token_embed"], g["token_embed"][0]) == 0.0
    assert rel_max(dbg["prelookahead"], g["prelookahead"][0]) < 1e-5
    assert rel_max(dbg["mu"], g["mu"][0]) < 1e-5
    assert rel_max(dbg["cond"], g["cond"][0]) < 1e-6
    assert rel_max(dbg["time_embed"], g["time_embed_step1"]) < 1e-5
    for i in (0, 10, 21):
        assert rel_max(dbg["blocks"][i], g[f"dit_block{i}"]) < STAGE_TOL
    cap = {}
    fo.infer(weights, g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0], g["spk_embedding"][0],
             g["noise_z"][0], capture=cap)
    for i in range(22):
        assert rel_max(dbg["blocks"][i], cap["blocks"][i]) < STAGE_TOL, i


def test_decode_chunked_vs_oracle(dec, weights):
    """Block-causal (chunk 50) 10-step CFG decode of two streams vs the oracle."""
    rng = np.random.default_rng(4)
    L = [56, 106]
    mus = [rng.standard_normal((80, n)).astype(np.float32) for n in L]
    conds = [np.zeros((80, n), np.float32) for n in L]
    noise = [rng.standard_normal((80, n)).astype(np.float32) for n in L]
    spks = rng.standard_normal((2, 80)).astype(np.float32)
    out = dec.decode(L, mus, conds, spks, noise=noise, chunk=50)
    for b, n in enumerate(L):
        ref = fo.solve_euler(weights, noise[b][None], mus[b][None], spks[b:b + 1], conds[b][None],
                             fo.block_causal_mask([n], n, 50))[0]
        assert np.abs(_split(out, L)[b] - ref).max() < MEL_ABS_TOL


def test_errors_are_reported(dec, tmp_path):
    """Bad inputs fail with a status, not a crash."""
    from larynx_b200 import FlowDecoder
    d = FlowDecoder(0)
    assert not d.load(str(tmp_path / "missing.gguf"))
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\0" * 64)
    assert not d.load(str(bad))
    assert "infer" and d.infer([1], [2], np.zeros((0, 80)), np.ones(192)) is None  # not loaded
    d.close()
    with pytest.raises(Exception):
        dec.decode([0], np.zeros(0), np.zeros(0), np.zeros((1, 80)), noise=np.zeros(0))


def test_noise_bank_production_path(dec, tmp_path):
    """The 6-argument FlowDecoder::infer (flow.h:72-77, flow.cpp:290-308): the
    CFM noise is the first MEL_T columns of the bank given to load_noise
    (FNSE asset, flow.cpp:70-108).  It must equal the 7-argument call fed
    that slice, bit for bit; so must the batched decode with noise=None."""
    import struct

    from larynx_b200.gguf import write_noise_bank
    rng = np.random.default_rng(21)
    bank = rng.standard_normal((80, 15000), dtype=np.float32)
    path = str(tmp_path / "flow_noise.bin")
    write_noise_bank(path, bank)
    assert dec.load_noise(path), dec.last_error
    g = golden("flow_fixture.npz")
    args = (g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0], g["spk_embedding"][0])
    T = 2 * (g["prompt_tokens"].size + g["tokens"].size)
    a = dec.infer(*args)                                  # bank slice
    b = dec.infer(*args, noise_z=bank[:, :T])             # explicit noise
    assert a is not None and b is not None
    np.testing.assert_array_equal(a, b)
    # batched decode: noise=None slices the bank per utterance
    L = [40, 17]
    mus = [rng.standard_normal((80, n)).astype(np.float32) for n in L]
    conds = [np.zeros((80, n), np.float32) for n in L]
    spks = rng.standard_normal((2, 80)).astype(np.float32)
    d0 = dec.decode(L, mus, conds, spks, noise=None)
    d1 = dec.decode(L, mus, conds, spks, noise=[bank[:, :n] for n in L])
    np.testing.assert_array_equal(d0, d1)

    # idempotent like the reference (flow.cpp:72): a loaded bank stays loaded
    assert dec.load_noise(str(tmp_path / "missing.bin"))
    np.testing.assert_array_equal(dec.infer(*args), a)

    # malformed assets are rejected with a status, on a handle with no bank yet
    from larynx_b200 import FlowDecoder
    fresh = FlowDecoder(0)

    def bad(name, header, payload_floats):
        p = str(tmp_path / name)
        with open(p, "wb") as f:
            f.write(header)
            f.write(np.zeros(payload_floats, np.float32).tobytes())
        return p
    n = 80 * 15000
    for p in (bad("magic.bin", struct.pack("<IIIQ", 0x12345678, 1, 80, 15000), n),
              bad("version.bin", struct.pack("<IIIQ", 0x45534E46, 2, 80, 15000), n),
              bad("mel.bin", struct.pack("<IIIQ", 0x45534E46, 1, 81, 15000), n),
              bad("frames.bin", struct.pack("<IIIQ", 0x45534E46, 1, 80, 14999), n),
              bad("short.bin", struct.pack("<IIIQ", 0x45534E46, 1, 80, 15000), n - 1),
              str(tmp_path / "missing.bin")):
        assert not fresh.load_noise(p), p
        assert fresh.last_error
    assert fresh.load_noise(path), fresh.last_error
    fresh.close()


def test_decode_after_workspace_growth_matches_fresh_handle(dec, gguf_path):
    """A handle whose workspace grew (a small batch, then one that needs more
    rows: every buffer and tensor map is reallocated) decodes the larger
    batch bit for bit as a fresh handle does.  The rows past the last packed
    row of each plan are never read as valid data (the sequence of the
    multi-GPU bench: shards, then the 20 s utterance, then the whole set)."""
    from larynx_b200 import FlowDecoder
    rng = np.random.default_rng(11)

    def batch(lengths):
        mus = [rng.standard_normal((80, n)).astype(np.float32) for n in lengths]
        conds = [np.where(np.arange(n) < n // 5, rng.standard_normal((80, n)), 0).astype(np.float32)
                 for n in lengths]
        noise = [rng.standard_normal((80, n)).astype(np.float32) for n in lengths]
        spks = rng.standard_normal((len(lengths), 80)).astype(np.float32)
        return mus, conds, spks, noise

    small = [131, 77, 250]
    large = [1000, 333, 1499, 517, 64, 1201, 250, 903]  # > 4096 and > 9.5k packed rows: pair GEMMs
    s_args = batch(small)
    l_args = batch(large)
    fresh = FlowDecoder(0)
    assert fresh.load(gguf_path), fresh.last_error
    want = fresh.decode(large, *l_args[:3], noise=l_args[3])
    fresh.close()
    d = FlowDecoder(0)
    assert d.load(gguf_path), d.last_error
    d.decode(small, *s_args[:3], noise=s_args[3])
    d.decode([1000], *batch([1000])[:3], noise=batch([1000])[3])
    got = d.decode(large, *l_args[:3], noise=l_args[3])
    d.close()
    assert np.isfinite(got).all()
    assert np.array_equal(got, want)
