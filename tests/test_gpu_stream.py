"""The streaming call (finalize=False) and the chunked streaming driver on the
GPU, through the C ABI: parity with the reference's own streaming inference
(golden vectors from tests/flow_reference.py) and the driver's bookkeeping
against direct calls."""

import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu

MEL_ABS_TOL = 2e-2   # final mel max-abs after 10 steps (north star)


@pytest.fixture(scope="module")
def dec(tmp_path_factory):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    from larynx_b200 import FlowDecoder
    from larynx_b200.weights import write_synthetic_gguf
    p = str(tmp_path_factory.mktemp("w") / "flow_synth.gguf")
    write_synthetic_gguf(p, seed=0, std=0.02)
    d = FlowDecoder(0)
    assert d.load(p), d.last_error
    yield d
    d.close()


def test_streaming_call_golden(dec):
    g = golden("flow_stream.npz")
    args = (g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0], g["spk_embedding"][0])
    dbg_s = {}
    mel_s = dec.infer(*args, noise_z=g["noise_z"][0], finalize=False, debug=dbg_s)
    assert mel_s is not None and mel_s.shape == g["feat_stream"][0].shape
    assert np.abs(mel_s - g["feat_stream"][0]).max() < MEL_ABS_TOL
    # the streaming PreLookahead (last 3 tokens as context): 16 tokens in, 13 rows out
    assert dbg_s["token_embed"].shape == (16, 80)
    assert dbg_s["prelookahead"].shape == g["prelookahead"][0].shape
    assert np.abs(dbg_s["prelookahead"] - g["prelookahead"][0]).max() < 1e-5 * np.abs(g["prelookahead"]).max()
    dbg = {}
    mel_f = dec.infer(*args, noise_z=g["noise_z"][0], finalize=True, debug=dbg)
    assert np.abs(mel_f - g["feat_final"][0]).max() < MEL_ABS_TOL
    # the two calls see different PreLookahead inputs for the last frames
    assert np.abs(mel_f[:, :mel_s.shape[1]] - mel_s).max() > 1e-3


def test_streaming_call_needs_lookahead(dec):
    # 3 tokens in all: every one of them is look-ahead context, no frame to make
    out = dec.infer([1, 2], [3], np.zeros((0, 80), np.float32), np.ones(192, np.float32),
                    noise_z=np.zeros((80, 8), np.float32), finalize=False)
    assert out is None and dec.last_error


@pytest.mark.parametrize("chunk", [0, 50])
def test_streamer_matches_direct_calls(dec, chunk):
    from larynx_b200.stream import FlowStreamer
    rng = np.random.default_rng(7)
    P, N = 4, 83
    prompt = rng.integers(0, 6561, P)
    toks = rng.integers(0, 6561, N)
    pf = rng.standard_normal((2 * P, 80)).astype(np.float32)
    spk = rng.standard_normal(192).astype(np.float32)
    noise = rng.standard_normal((80, 2 * (P + N))).astype(np.float32)
    st = FlowStreamer(dec, prompt, pf, spk, noise_z=noise, hop=25, chunk=chunk)
    segs = []
    for i in range(0, N, 7):
        segs.append(st.push(toks[i:i + 7]))
    segs.append(st.finish())
    mel = np.concatenate(segs, axis=1)
    assert mel.shape == (80, 2 * N)
    # hops of 25 tokens emitted when 28 were available: 25, 50, 75 tokens
    assert st.emitted_tokens == 75 and st.calls == 4
    # every streamed segment equals the same slice of a direct call
    for k, upto in enumerate((25, 50, 75)):
        direct = dec.infer(prompt, toks[:upto + 3], pf, spk, noise_z=noise, finalize=False, chunk=chunk)
        np.testing.assert_array_equal(mel[:, 2 * (upto - 25):2 * upto], direct[:, 2 * (upto - 25):2 * upto])
    final = dec.infer(prompt, toks, pf, spk, noise_z=noise, finalize=True, chunk=chunk)
    np.testing.assert_array_equal(mel[:, 150:], final[:, 150:])
    assert np.isfinite(mel).all()
