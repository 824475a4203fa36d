"""Pins the HiFT oracle's host stages to the reference's own code.

oracle/_ref/libhift_source_ref.so is the reference's src/hift/source.cpp
(float64 f0 predictor, SineGen2 + m_source + STFT, ISTFT) compiled from its
own file by oracle/Makefile.  oracle/hift_oracle.py restates those functions
in the same operation order; here both run on the same seeded synthetic
weights and inputs: f0 must agree bit for bit, the float32 stages within a
few ulps (numpy's vectorised sin / cos / tanh may differ from libm's in the
last bit).  Skipped where the reference was not present to build the library.
"""

import ctypes
import os

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "oracle", "_ref", "libhift_source_ref.so")

pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="oracle/_ref not built (no reference checkout)")

_f64p = ctypes.POINTER(ctypes.c_double)
_f32p = ctypes.POINTER(ctypes.c_float)


@pytest.fixture(scope="module")
def ref():
    lib = ctypes.CDLL(LIB)
    lib.hiftref_f0_predict.argtypes = [_f64p, ctypes.c_int, ctypes.POINTER(_f64p), ctypes.POINTER(_f64p), _f64p, _f64p,
                                       _f64p]
    lib.hiftref_f0_predict.restype = None
    lib.hiftref_source_stft.argtypes = [_f32p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
    lib.hiftref_source_stft.restype = None
    lib.hiftref_istft.argtypes = [_f32p, _f32p, ctypes.c_int, _f32p]
    lib.hiftref_istft.restype = None
    return lib


@pytest.fixture(scope="module")
def w():
    from larynx_b200.hift_weights import synthetic_weights
    return synthetic_weights(0)


def _p(a, t):
    return a.ctypes.data_as(t)


def _ref_f0(ref, w, mel):
    T = mel.shape[1]
    ws = [np.ascontiguousarray(w[f"f0_predictor.condnet.{i}.weight"], np.float64) for i in (0, 2, 4, 6, 8)]
    bs = [np.ascontiguousarray(w[f"f0_predictor.condnet.{i}.bias"], np.float64) for i in (0, 2, 4, 6, 8)]
    wp = (_f64p * 5)(*[_p(a, _f64p) for a in ws])
    bp = (_f64p * 5)(*[_p(a, _f64p) for a in bs])
    cw = np.ascontiguousarray(w["f0_predictor.classifier.weight"].reshape(-1), np.float64)
    cb = np.ascontiguousarray(w["f0_predictor.classifier.bias"].reshape(-1), np.float64)
    m = np.ascontiguousarray(mel, np.float64)
    out = np.empty(T, np.float64)
    ref.hiftref_f0_predict(_p(m, _f64p), T, wp, bp, _p(cw, _f64p), _p(cb, _f64p), _p(out, _f64p))
    return out


@pytest.mark.parametrize("T", [1, 30, 157])
def test_f0_predictor_bit_exact(ref, w, T):
    from oracle import hift_oracle as ho
    mel = np.random.default_rng(T).standard_normal((80, T)).astype(np.float32)
    np.testing.assert_array_equal(ho.f0_predict(mel, w), _ref_f0(ref, w, mel))


@pytest.mark.parametrize("T", [1, 30])
def test_source_stft(ref, w, T):
    from larynx_b200.hift_weights import synthetic_source
    from oracle import hift_oracle as ho
    mel = np.random.default_rng(100 + T).standard_normal((80, T)).astype(np.float32)
    f0 = ho.f0_predict(mel, w).astype(np.float32)
    ri, bank = synthetic_source(0, T * 480)
    bank = np.ascontiguousarray(bank[:T * 480 * 9], np.float32).reshape(T * 480, 9)
    ri = np.ascontiguousarray(ri, np.float32)
    L_S = T * 480
    n_frames = L_S // 4 + 1
    st = np.empty((18, n_frames), np.float32)
    wavs = np.empty((L_S, 9), np.float32)
    merge = np.empty(L_S, np.float32)
    mw = np.ascontiguousarray(w["m_source.l_linear.weight"].reshape(-1), np.float32)
    mb = np.ascontiguousarray(w["m_source.l_linear.bias"].reshape(-1), np.float32)
    ref.hiftref_source_stft(_p(f0, _f32p), T, _p(ri, _f32p), _p(bank, _f32p), _p(mw, _f32p), _p(mb, _f32p),
                            _p(st, _f32p), _p(wavs, _f32p), _p(merge, _f32p))
    o_st, o_wavs, o_merge = ho.source_stft(f0, ri, bank, w)
    assert np.abs(o_wavs - wavs).max() <= 1e-6 * max(1.0, np.abs(wavs).max())
    assert np.abs(o_merge - merge).max() <= 1e-6
    assert np.abs(o_st - st).max() <= 1e-6 * max(1.0, np.abs(st).max())


@pytest.mark.parametrize("n_frames", [2, 361, 3601])
def test_istft(ref, n_frames):
    from oracle import hift_oracle as ho
    rng = np.random.default_rng(n_frames)
    mag = np.ascontiguousarray(np.abs(rng.standard_normal((9, n_frames))) * 3, np.float32)
    mag[0, 0] = 250.0            # above the 1e2 clip
    ph = np.ascontiguousarray(rng.uniform(-np.pi, np.pi, (9, n_frames)), np.float32)
    out = np.empty((n_frames - 1) * 4, np.float32)
    ref.hiftref_istft(_p(mag, _f32p), _p(ph, _f32p), n_frames, _p(out, _f32p))
    got = ho.istft(mag, ph)
    assert got.shape == out.shape
    assert np.abs(got - out).max() <= 1e-6 * max(1.0, np.abs(out).max())
