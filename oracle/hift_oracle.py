"""CPU oracle for the HiFT vocoder (TEST INFRASTRUCTURE ONLY).

The parity checker for the CUDA HiFT vocoder in ``larynx_b200``.  It restates,
in plain numpy, the reference's CausalHiFTGenerator (finalize=True path):

  * ``src/hift/source.cpp`` of hardenedlinux/larynx for the host stages: the
    float64 f0 predictor, SineGen2 + m_source + the 16-point STFT (float32),
    and the ISTFT -- in the same operation order, so float64 results are
    bit-identical and float32 ones differ only where numpy's sin/cos/tanh
    differ from the C library's by an ulp;
  * ``src/hift/hift.cpp:183-252`` and ``ops.cpp`` for the conv network
    (conv_pre, three upsample + source-fusion + resblock stages, conv_post,
    exp/sin split), float32, with ``docs/HIFT.md`` section 1 for the PyTorch
    semantics it reproduces (causal padding sides, Snake, the final
    leaky_relu slope 0.01, the magnitude clip at 1e2).

Parity unpinned: the reference's ground truth (``tests/hift_reference.py``)
imports the CosyVoice package, which is not in this checkout, and its C++
needs the GGML library; no golden vectors exist for this module.

Layouts follow the reference: channel-major [C][T] (PyTorch (1, C, T)).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this module.
"""

from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np

IN_CH = 80
BASE_CH = 512
NB_HARM = 8
SAMPLE_RATE = 24000
NSF_ALPHA = np.float32(0.1)
NSF_SIGMA = np.float32(0.003)
NSF_VOICED = np.float32(10.0)
UPSAMPLE_RATES = (8, 5, 3)
UPSAMPLE_KERNELS = (16, 11, 7)
ISTFT_N_FFT = 16
ISTFT_HOP = 4
N_BINS = 9
OUT_CH = 18
RESBLOCK_KERNELS = (3, 7, 11)
RESBLOCK_DILATIONS = (1, 3, 5)
SRC_RB_KERNELS = (7, 7, 11)
SRC_DOWN_KERNELS = (30, 6, 1)
SRC_DOWN_STRIDES = (15, 3, 1)
LRELU_SLOPE = np.float32(0.1)
AUDIO_LIMIT = np.float32(0.99)
CONV_PRE_LOOK_RIGHT = 4
TOTAL_SCALE = 8 * 5 * 3 * ISTFT_HOP  # 480
SNAKE_EPS = np.float32(1e-9)
F32 = np.float32


def stage_channels(i: int) -> int:
    return BASE_CH >> (i + 1)


# ---------------------------------------------------------------------------
# f0 predictor, float64 (source.cpp:18-40, 70-96)
# ---------------------------------------------------------------------------
def _conv1d_s1_f64(x: np.ndarray, W: np.ndarray, b: np.ndarray, pad_left: int) -> np.ndarray:
    """source.cpp:18-35: out[oc][t] = b[oc] + sum_ic sum_k W[oc][ic][k] x[ic][t+k-pad_left]
    (zero outside), accumulated ic-major then k, one product at a time."""
    IC, L = x.shape
    OC, _, K = W.shape
    xp = np.zeros((IC, L + K), np.float64)
    xp[:, pad_left:pad_left + L] = x
    acc = np.repeat(b.astype(np.float64)[:, None], L, axis=1)
    for ic in range(IC):
        for k in range(K):
            acc += W[:, ic, k].astype(np.float64)[:, None] * xp[ic, k:k + L][None, :]
    return acc


_libm_exp = np.frompyfunc(math.exp, 1, 1)


def _elu(v: np.ndarray) -> np.ndarray:
    """source.cpp:38-40: x <= 0 -> std::exp(x) - 1.  The exponential is the C
    library's (Python's math.exp): numpy's vectorised float64 exp differs from
    it in the last bit for some inputs, which the reference's own compiled
    source.cpp (oracle/_ref) shows."""
    out = np.array(v, np.float64, copy=True)
    neg = out <= 0.0
    out[neg] = _libm_exp(out[neg]).astype(np.float64) - 1.0
    return out


def f0_predict(mel: np.ndarray, w: Dict[str, np.ndarray]) -> np.ndarray:
    """mel [80][T] -> f0 [T] float64 (source.cpp:70-96)."""
    x = np.asarray(mel, np.float64)
    y = _elu(_conv1d_s1_f64(x, w["f0_predictor.condnet.0.weight"], w["f0_predictor.condnet.0.bias"], 0))
    for idx in (2, 4, 6, 8):
        y = _elu(_conv1d_s1_f64(y, w[f"f0_predictor.condnet.{idx}.weight"], w[f"f0_predictor.condnet.{idx}.bias"], 2))
    cw = w["f0_predictor.classifier.weight"].astype(np.float64).reshape(-1)
    acc = np.full(y.shape[1], float(w["f0_predictor.classifier.bias"].reshape(-1)[0]), np.float64)
    for ic in range(BASE_CH):
        acc += cw[ic] * y[ic]
    return np.abs(acc)


# ---------------------------------------------------------------------------
# STFT helpers (source.cpp:46-67)
# ---------------------------------------------------------------------------
def hann_window() -> np.ndarray:
    n = np.arange(ISTFT_N_FFT, dtype=np.float32)
    arg = (F32(2.0) * F32(math.pi) * n) / F32(ISTFT_N_FFT)
    return (F32(0.5) * (F32(1.0) - np.cos(arg).astype(np.float32))).astype(np.float32)


def dft_tables():
    f = np.arange(ISTFT_N_FFT)[:, None].astype(np.float64)
    n = np.arange(ISTFT_N_FFT)[None, :].astype(np.float64)
    a = 2.0 * math.pi * f * n / ISTFT_N_FFT
    return np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)


# ---------------------------------------------------------------------------
# SineGen2 + m_source + STFT, float32 (source.cpp:98-196)
# ---------------------------------------------------------------------------
def source_stft(f0: np.ndarray, rand_ini: np.ndarray, sine_waves: np.ndarray, w: Dict[str, np.ndarray]):
    """f0 [T] float32 -> (s_stft [18][N_FRAMES], sine_wavs [L_S][9], sine_merge [L_S])."""
    f0 = np.asarray(f0, np.float32)
    T = f0.shape[0]
    L_S = T * TOTAL_SCALE
    n_frames = L_S // ISTFT_HOP + 1
    H = NB_HARM + 1
    f0up = np.repeat(f0, TOTAL_SCALE)
    fn = f0up[:, None] * np.arange(1, H + 1, dtype=np.float32)[None, :]
    rad = np.fmod(fn / F32(SAMPLE_RATE), F32(1.0)).astype(np.float32)
    rad[0] = rad[0] + np.asarray(rand_ini, np.float32)
    # linear x(1/480) downsample, align_corners=False (source.cpp:117-129)
    i = np.arange(T, dtype=np.float32)
    src = (i + F32(0.5)) * F32(L_S // T) - F32(0.5)
    fl = np.floor(src).astype(np.int64)
    cl = np.minimum(fl + 1, L_S - 1)
    frac = (src - fl.astype(np.float32)).astype(np.float32)
    rad_down = rad[fl] * (F32(1.0) - frac)[:, None] + rad[cl] * frac[:, None]
    cums = np.cumsum(rad_down.astype(np.float32), axis=0, dtype=np.float32)
    p = cums[np.arange(L_S) // TOTAL_SCALE]
    p = p * F32(2.0)
    p = p * F32(math.pi)
    p = p * F32(TOTAL_SCALE)
    s = np.sin(p).astype(np.float32) * NSF_ALPHA
    uv = (f0up > NSF_VOICED).astype(np.float32)[:, None]
    noise_amp = uv * NSF_SIGMA + ((F32(1.0) - uv) * NSF_ALPHA) / F32(3.0)
    noise = noise_amp * np.asarray(sine_waves, np.float32).reshape(L_S, H)
    sine_wavs = (s * uv + noise).astype(np.float32)
    mw = w["m_source.l_linear.weight"].reshape(-1).astype(np.float32)
    acc = np.full(L_S, w["m_source.l_linear.bias"].reshape(-1)[0], np.float32)
    for h in range(H):
        acc = acc + mw[h] * sine_wavs[:, h]
    sm = np.tanh(acc).astype(np.float32)
    # STFT: center reflect-pad 8, periodic Hann, onesided 9 bins
    pad = ISTFT_N_FFT // 2
    xp = np.concatenate([sm[1:pad + 1][::-1], sm, sm[L_S - 1 - pad:L_S - 1][::-1]]).astype(np.float32)
    win = hann_window()
    c, sn = dft_tables()
    idx = np.arange(n_frames)[:, None] * ISTFT_HOP + np.arange(ISTFT_N_FFT)[None, :]
    seg = xp[idx] * win[None, :]
    re = np.zeros((N_BINS, n_frames), np.float32)
    im = np.zeros((N_BINS, n_frames), np.float32)
    for n in range(ISTFT_N_FFT):
        re = re + seg[None, :, n] * c[:N_BINS, n][:, None]
        im = im - seg[None, :, n] * sn[:N_BINS, n][:, None]
    return np.concatenate([re, im], axis=0), sine_wavs, sm


def istft(magnitude: np.ndarray, phase: np.ndarray) -> np.ndarray:
    """magnitude/phase [9][N_FRAMES] -> raw audio [(N_FRAMES-1)*4] (source.cpp:198-239)."""
    n_frames = magnitude.shape[1]
    L_S = (n_frames - 1) * ISTFT_HOP
    m = np.minimum(magnitude.astype(np.float32), F32(100.0))
    Xr = np.zeros((ISTFT_N_FFT, n_frames), np.float32)
    Xi = np.zeros((ISTFT_N_FFT, n_frames), np.float32)
    Xr[:N_BINS] = m * np.cos(phase.astype(np.float32))
    Xi[:N_BINS] = m * np.sin(phase.astype(np.float32))
    for k in range(1, ISTFT_N_FFT // 2):
        Xr[ISTFT_N_FFT - k] = Xr[k]
        Xi[ISTFT_N_FFT - k] = -Xi[k]
    c, sn = dft_tables()
    win = hann_window()
    v = np.zeros((ISTFT_N_FFT, n_frames), np.float32)
    for k in range(ISTFT_N_FFT):
        v = v + (Xr[k][None, :] * c[k][:, None] - Xi[k][None, :] * sn[k][:, None])
    v = v / F32(ISTFT_N_FFT)
    out_len = L_S + ISTFT_N_FFT
    acc = np.zeros(out_len, np.float32)
    env = np.zeros(out_len, np.float32)
    t4 = np.arange(n_frames) * ISTFT_HOP
    # frames in increasing order reach a sample with decreasing n
    for n in range(ISTFT_N_FFT - 1, -1, -1):
        acc[t4 + n] += v[n] * win[n]
        env[t4 + n] += win[n] * win[n]
    e = np.maximum(env[ISTFT_N_FFT // 2:ISTFT_N_FFT // 2 + L_S], F32(1e-8))
    return (acc[ISTFT_N_FFT // 2:ISTFT_N_FFT // 2 + L_S] / e).astype(np.float32)


# ---------------------------------------------------------------------------
# Conv network, float32 (hift.cpp:22-40, 183-252; ops.cpp)
# ---------------------------------------------------------------------------
def conv1d(x: np.ndarray, W: np.ndarray, b: Optional[np.ndarray], stride: int = 1, dil: int = 1,
           pad_left: int = 0, pad_right: int = 0) -> np.ndarray:
    """Conv1d over [IC][L] with explicit zero padding (ops.cpp conv1d_f32 after
    pad_zeros): out[oc][t] = b[oc] + sum_{ic,k} W[oc][ic][k] xp[ic][t*stride + k*dil]."""
    x = np.asarray(x, np.float32)
    IC, L = x.shape
    OC, _, K = W.shape
    xp = np.zeros((IC, L + pad_left + pad_right), np.float32)
    xp[:, pad_left:pad_left + L] = x
    L_out = (xp.shape[1] - dil * (K - 1) - 1) // stride + 1
    cols = np.empty((IC, K, L_out), np.float32)
    for k in range(K):
        cols[:, k, :] = xp[:, k * dil: k * dil + stride * (L_out - 1) + 1: stride]
    out = W.reshape(OC, IC * K).astype(np.float32) @ cols.reshape(IC * K, L_out)
    if b is not None:
        out = out + b.astype(np.float32)[:, None]
    return out.astype(np.float32)


def snake(x: np.ndarray, alpha: np.ndarray) -> np.ndarray:
    """x + 1/(alpha + 1e-9) * sin(x alpha)^2, per channel (ops.cpp snake)."""
    a = alpha.astype(np.float32)[:, None]
    inv = (F32(1.0) / (alpha.astype(np.float32) + SNAKE_EPS))[:, None]
    s = np.sin(x * a).astype(np.float32)
    return (x + inv * (s * s)).astype(np.float32)


def leaky_relu(x: np.ndarray, slope) -> np.ndarray:
    return np.where(x > 0, x, x * F32(slope)).astype(np.float32)


def resblock(x: np.ndarray, w: Dict[str, np.ndarray], prefix: str, k: int) -> np.ndarray:
    """hift.cpp:25-40: 3 x (snake1 -> conv1(dilation d_j) -> snake2 -> conv2) + residual."""
    for j in range(3):
        d = RESBLOCK_DILATIONS[j]
        xt = snake(x, w[f"{prefix}.activations1.{j}.alpha"])
        xt = conv1d(xt, w[f"{prefix}.convs1.{j}.weight"], w[f"{prefix}.convs1.{j}.bias"], dil=d, pad_left=d * (k - 1))
        xt = snake(xt, w[f"{prefix}.activations2.{j}.alpha"])
        xt = conv1d(xt, w[f"{prefix}.convs2.{j}.weight"], w[f"{prefix}.convs2.{j}.bias"], pad_left=k - 1)
        x = (xt + x).astype(np.float32)
    return x


def decode(mel: np.ndarray, s_stft: np.ndarray, w: Dict[str, np.ndarray], cap: Optional[dict] = None):
    """mel [80][T], s_stft [18][N_FRAMES] -> (magnitude, phase) [9][N_FRAMES]."""
    cap = cap if cap is not None else {}
    x = conv1d(mel, w["conv_pre.weight"], w["conv_pre.bias"], pad_right=CONV_PRE_LOOK_RIGHT)
    cap["conv_pre"] = x
    for i in range(3):
        x = leaky_relu(x, LRELU_SLOPE)
        cap[f"ups{i}_lrelu"] = x
        u = np.repeat(x, UPSAMPLE_RATES[i], axis=1)
        x = conv1d(u, w[f"ups.{i}.weight"], w[f"ups.{i}.bias"], pad_left=UPSAMPLE_KERNELS[i] - 1)
        cap[f"ups{i}"] = x
        if i == 2:
            x = np.concatenate([x[:, 1:2], x], axis=1)
            cap["reflection_pad"] = x
        st = SRC_DOWN_STRIDES[i]
        if st == 1:
            si = conv1d(s_stft, w[f"source_downs.{i}.weight"], w[f"source_downs.{i}.bias"])
        else:
            si = conv1d(s_stft, w[f"source_downs.{i}.weight"], w[f"source_downs.{i}.bias"], stride=st,
                        pad_left=st - 1)
        cap[f"source_downs{i}"] = si
        si = resblock(si, w, f"source_resblocks.{i}", SRC_RB_KERNELS[i])
        cap[f"source_resblocks{i}"] = si
        x = (x + si).astype(np.float32)
        cap[f"fusion{i}"] = x
        xs = None
        for j in range(3):
            r = resblock(x, w, f"resblocks.{i * 3 + j}", RESBLOCK_KERNELS[j])
            cap[f"resblock{i * 3 + j}"] = r
            xs = r if xs is None else (xs + r).astype(np.float32)
        x = (xs * F32(1.0 / 3.0)).astype(np.float32)
        cap[f"post_resblocks{i}"] = x
    x = leaky_relu(x, 0.01)
    cap["final_lrelu"] = x
    x = conv1d(x, w["conv_post.weight"], w["conv_post.bias"], pad_left=6)
    cap["conv_post"] = x
    magnitude = np.exp(x[:N_BINS]).astype(np.float32)
    phase = np.sin(x[N_BINS:]).astype(np.float32)
    return magnitude, phase


def vocode(mel: np.ndarray, rand_ini: np.ndarray, sine_waves: np.ndarray, w: Dict[str, np.ndarray],
           cap: Optional[dict] = None) -> np.ndarray:
    """HiftVocoder::vocode (hift.cpp:140-303): mel [80][T] -> audio [T*480]."""
    cap = cap if cap is not None else {}
    mel = np.asarray(mel, np.float32).reshape(IN_CH, -1)
    T = mel.shape[1]
    f0 = f0_predict(mel, w).astype(np.float32)
    cap["f0"] = f0
    s_stft, sine_wavs, sine_merge = source_stft(f0, rand_ini, np.asarray(sine_waves, np.float32)[:T * TOTAL_SCALE], w)
    cap["sine_wavs"], cap["sine_merge"], cap["s_stft"] = sine_wavs, sine_merge, s_stft
    magnitude, phase = decode(mel, s_stft, w, cap)
    cap["magnitude"], cap["phase"] = magnitude, phase
    raw = istft(magnitude, phase)
    cap["istft"] = raw
    audio = np.clip(raw, -AUDIO_LIMIT, AUDIO_LIMIT).astype(np.float32)
    cap["speech"] = audio
    return audio
