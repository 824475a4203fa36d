"""The numpy oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py ran hardenedlinux/larynx's tests/flow_reference.py
on the same seeded synthetic weights).  These pin the oracle before it is used
to judge the CUDA path."""

import numpy as np
import pytest

from conftest import golden, rel_max
from oracle import flow_oracle as fo

TOL = 2e-5   # float32 vs float32 (torch BLAS/SDPA vs numpy BLAS): accumulation noise


def test_ops_fixture(weights):
    g = golden("ops_fixture.npz")
    x, mod = g["x"], g["mod"]
    D = 1024
    got = fo.op_adaln_mod(x, mod[0, :D], mod[0, D:2 * D])
    assert rel_max(got, g["adaln"]) < TOL
    assert rel_max(fo.op_rotary(x, g["pos"]), g["rotary"]) < TOL
    assert rel_max(fo.gelu_tanh(x * np.float32(3)), g["gelu"]) < TOL
    assert rel_max(fo.mish(x * np.float32(3)), g["mish"]) < TOL
    np.testing.assert_allclose(fo.t_span_cosine(), g["t_span"], atol=1e-7)
    temb = fo.time_embed(weights, g["t_span"][:10])
    assert rel_max(temb, g["temb"]) < TOL
    assert rel_max(np.concatenate(fo.adaln_chunks(weights, 0, temb), -1), g["mod_block0"]) < TOL
    assert rel_max(np.concatenate(fo.final_chunks(weights, temb), -1), g["mod_final"]) < TOL


def test_flow_fixture_stages(weights):
    """The reference's own 24-frame validation case, stage by stage."""
    g = golden("flow_fixture.npz")
    cap = {}
    mel = fo.infer(weights, g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0],
                   g["spk_embedding"][0], g["noise_z"][0], capture=cap)
    assert rel_max(cap["spk"], g["spk"][0]) < TOL
    assert rel_max(cap["token_embed"], g["token_embed"][0]) < TOL
    assert rel_max(cap["prelookahead"], g["prelookahead"][0]) < TOL
    assert rel_max(cap["time_embed"], g["time_embed_step1"]) < TOL
    assert rel_max(cap["input_proj"], g["dit_input_proj_step1"]) < TOL
    assert rel_max(cap["conv_pos"], g["dit_conv_pos_step1"]) < TOL
    assert rel_max(cap["input_embed"], g["dit_input_embed_step1"]) < TOL
    for i in (0, 10, 21):
        assert rel_max(cap["blocks"][i], g[f"dit_block{i}"]) < TOL, i
    assert rel_max(cap["norm_out"], g["dit_norm_out_step1"]) < TOL
    assert rel_max(cap["dphi_step1"], g["dphi_step1"]) < TOL
    assert rel_max(mel, g["feat"][0]) < TOL


def test_padded_batch(weights):
    """Key-padding mask: valid frames of a padded batch (one forward and a
    10-step CFG solve) match the reference."""
    g = golden("dit_padded.npz")
    L = g["lengths"]
    T = int(L.max())
    mask = fo.key_padding_mask(L, T)
    d = fo.dit_forward(weights, g["x"], g["mu"], np.full(len(L), g["t"], np.float32), g["spks"], g["cond"], mask)
    for b, n in enumerate(L):
        assert rel_max(d[b, :, :n], g["dphi"][b, :, :n]) < TOL
    xs = fo.solve_euler(weights, g["x"], g["mu"], g["spks"], g["cond"], mask)
    for b, n in enumerate(L):
        assert rel_max(xs[b, :, :n], g["solve"][b, :, :n]) < TOL


def test_padded_equals_solo(weights):
    """Valid frames of a padded batch equal a solo unpadded run."""
    g = golden("dit_padded.npz")
    L = g["lengths"]
    T = int(L.max())
    d = fo.dit_forward(weights, g["x"], g["mu"], np.full(len(L), g["t"], np.float32), g["spks"], g["cond"],
                       fo.key_padding_mask(L, T))
    b, n = 0, int(L[0])
    solo = fo.dit_forward(weights, g["x"][b:b + 1, :, :n], g["mu"][b:b + 1, :, :n], np.full(1, g["t"], np.float32),
                          g["spks"][b:b + 1], g["cond"][b:b + 1, :, :n], None)
    assert rel_max(d[b, :, :n], solo[0]) < TOL


def test_block_causal_chunk(weights):
    g = golden("dit_chunk.npz")
    L = g["lengths"]
    T = int(L.max())
    mask = fo.block_causal_mask(L, T, int(g["chunk"]))
    d = fo.dit_forward(weights, g["x"], g["mu"], np.full(len(L), g["t"], np.float32), g["spks"], g["cond"], mask)
    for b, n in enumerate(L):
        assert rel_max(d[b, :, :n], g["dphi"][b, :, :n]) < TOL


def test_euler_schedule():
    sched = fo.euler_schedule()
    ts = fo.t_span_cosine()
    assert len(sched) == 10
    assert sched[0] == (0.0, float(ts[1]))
    assert abs(sum(dt for _, dt in sched) - 1.0) < 1e-6


def test_streaming_call(weights):
    """finalize=False: PreLookahead with the last 3 tokens as context
    (flow_reference.py:546-548); also the finalize=True output of the same
    inputs, which must differ from it."""
    g = golden("flow_stream.npz")
    cap = {}
    args = (g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0], g["spk_embedding"][0], g["noise_z"][0])
    mel_s = fo.infer(weights, *args, capture=cap, finalize=False)
    assert rel_max(cap["prelookahead"], g["prelookahead"][0]) < TOL
    assert mel_s.shape == g["feat_stream"][0].shape
    assert rel_max(mel_s, g["feat_stream"][0]) < TOL
    mel_f = fo.infer(weights, *args, finalize=True)
    assert rel_max(mel_f, g["feat_final"][0]) < TOL
    assert mel_f.shape[1] == mel_s.shape[1] + 2 * fo.PRE_LOOKAHEAD
    assert np.abs(mel_f[:, :mel_s.shape[1]] - mel_s).max() > 1e-3   # the look-ahead context changes the result
