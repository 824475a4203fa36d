"""CPU checks of the HiFT vocoder boundary and oracle: the library exports
every symbol include/larynx_hift.h declares; the synthetic hift.gguf carries
the reference's 246-tensor inventory; the source asset has the HSRC layout;
creating a vocoder without an sm_100 GPU fails loudly; and size-independent
properties of the oracle (STFT -> ISTFT reconstruction, the f0 predictor's
ordered float64 conv against a plain convolution, the float32 conv against a
direct loop)."""

import os
import re
import struct

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(REPO, "include", "larynx_hift.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|void|const char\*)\s+(lx_hift_\w+)\s*\(", src, re.M)))


def test_header_and_library_exports():
    import ctypes
    from larynx_b200.flow import load_library
    from larynx_b200.hift import HIFT_EXPORTS
    assert set(HIFT_EXPORTS) == set(_declared())
    lib = load_library()
    for s in HIFT_EXPORTS:
        assert ctypes.cast(getattr(lib, s), ctypes.c_void_p).value, s


def test_no_cpu_fallback_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from larynx_b200.hift import HiftError, HiftVocoder
    with pytest.raises(HiftError):
        HiftVocoder(0)


def test_synthetic_gguf_inventory(tmp_path):
    from larynx_b200.gguf import read_gguf_index
    from larynx_b200.hift_weights import param_specs, write_synthetic_hift_gguf
    p = str(tmp_path / "hift.gguf")
    write_synthetic_hift_gguf(p, seed=0)
    idx = read_gguf_index(p)
    specs = dict(param_specs())
    assert len(idx) == 246 == len(specs)
    for name, (shape, dtype) in idx.items():
        assert tuple(shape) == specs[name] and dtype == 0, name
    # the names the reference's loader resolves (src/hift/gguf.cpp:95-128)
    for n in ("conv_pre.weight", "ups.2.bias", "source_downs.0.weight", "source_resblocks.2.activations2.1.alpha",
              "resblocks.8.convs1.2.weight", "m_source.l_linear.weight", "f0_predictor.condnet.8.bias",
              "f0_predictor.classifier.weight"):
        assert n in idx


def test_source_asset_layout(tmp_path):
    from larynx_b200.hift_weights import write_source_asset
    ri = np.arange(9, dtype=np.float32)
    bank = np.arange(5 * 9, dtype=np.float32).reshape(5, 9)
    p = str(tmp_path / "src.bin")
    write_source_asset(p, ri, bank)
    raw = open(p, "rb").read()
    magic, ver, dim, smax = struct.unpack("<IIIQ", raw[:20])
    assert (magic, ver, dim, smax) == (0x43525348, 1, 9, 5)
    assert np.array_equal(np.frombuffer(raw[20:56], np.float32), ri)
    assert np.array_equal(np.frombuffer(raw[56:], np.float32).reshape(5, 9), bank)


def test_stft_istft_reconstruction():
    # a Hann window at hop 4 / n_fft 16 overlap-adds to a constant; with the
    # envelope normalisation the onesided STFT inverts exactly (to rounding)
    from oracle import hift_oracle as H
    rng = np.random.default_rng(5)
    T = 7
    L_S = T * H.TOTAL_SCALE
    s = rng.uniform(-0.5, 0.5, L_S).astype(np.float32)
    pad = 8
    xp = np.concatenate([s[1:pad + 1][::-1], s, s[L_S - 1 - pad:L_S - 1][::-1]])
    win = H.hann_window()
    n_frames = L_S // 4 + 1
    idx = np.arange(n_frames)[:, None] * 4 + np.arange(16)[None, :]
    X = np.fft.rfft(xp[idx].astype(np.float64) * win, axis=1).T  # [9][N]
    mag = np.abs(X).astype(np.float32)
    pha = np.angle(X).astype(np.float32)
    rec = H.istft(mag, pha)
    assert rec.shape == (L_S,)
    assert np.abs(rec - s).max() < 1e-5


def test_f0_conv_order_matches_plain_convolution():
    from oracle import hift_oracle as H
    rng = np.random.default_rng(2)
    x = rng.standard_normal((6, 11))
    W = rng.standard_normal((4, 6, 3))
    b = rng.standard_normal(4)
    got = H._conv1d_s1_f64(x, W, b, pad_left=2)
    want = np.zeros((4, 11))
    for oc in range(4):
        for t in range(11):
            acc = b[oc]
            for ic in range(6):
                for k in range(3):
                    src = t + k - 2
                    if 0 <= src < 11:
                        acc += W[oc, ic, k] * x[ic, src]
            want[oc, t] = acc
    assert np.array_equal(got, want)  # same order: bit-identical


def test_conv1d_against_direct_loop():
    from oracle import hift_oracle as H
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 40)).astype(np.float32)
    W = rng.standard_normal((3, 5, 6)).astype(np.float32)
    b = rng.standard_normal(3).astype(np.float32)
    for stride, dil, pl, pr in ((1, 1, 5, 0), (1, 3, 15, 0), (3, 1, 2, 0), (1, 1, 0, 4)):
        got = H.conv1d(x, W, b, stride=stride, dil=dil, pad_left=pl, pad_right=pr)
        xp = np.pad(x.astype(np.float64), ((0, 0), (pl, pr)))
        L_out = (xp.shape[1] - dil * 5 - 1) // stride + 1
        want = np.zeros((3, L_out))
        for t in range(L_out):
            for k in range(6):
                want[:, t] += W[:, :, k].astype(np.float64) @ xp[:, t * stride + k * dil]
        want += b[:, None]
        assert got.shape == want.shape
        assert np.abs(got - want).max() < 1e-4


def test_oracle_vocode_shapes_and_limits():
    from larynx_b200.hift_weights import synthetic_source, synthetic_weights
    from oracle import hift_oracle as H
    w = synthetic_weights(0)
    ri, bank = synthetic_source(0, 12 * 480)
    mel = np.random.default_rng(9).standard_normal((80, 12)).astype(np.float32)
    cap = {}
    audio = H.vocode(mel, ri, bank, w, cap)
    assert audio.shape == (12 * 480,) and np.isfinite(audio).all()
    assert np.abs(audio).max() <= 0.99
    assert cap["s_stft"].shape == (18, 12 * 120 + 1) and cap["reflection_pad"].shape == (64, 12 * 120 + 1)
    # voiced and unvoiced frames both occur with the synthetic weights
    assert 0 < (cap["f0"] > 10).sum() <= 12
