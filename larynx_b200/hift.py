"""Python host side of the B200 HiFT vocoder: a ctypes binding of the C ABI
(include/larynx_hift.h) that mirrors larynx's ``HiftVocoder``
(include/larynx/hift/hift.h:46-93): ``load``, ``load_source`` and ``vocode``
keep the reference's names, argument meaning and bool / None-on-failure
behaviour (errors are also printed to stderr).  ``vocode_device`` extends it
with device buffers on a caller stream.

Shares liblarynx_flow.so with the Flow decoder; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import sys
from typing import Optional

import numpy as np

from .flow import ERRORS, LX_OK, load_library

SAMPLES_PER_FRAME = 480
HARMONICS = 9
SINE_MAX_SAMPLES = 300 * 24000

HIFT_EXPORTS = ("lx_hift_create", "lx_hift_destroy", "lx_hift_last_error", "lx_hift_load_gguf",
                "lx_hift_load_source", "lx_hift_vocode", "lx_hift_vocode_device")

_f32p = ctypes.POINTER(ctypes.c_float)


class LxHiftDebug(ctypes.Structure):
    _fields_ = ([(n, _f32p) for n in ("f0", "sine_wavs", "sine_merge", "s_stft", "conv_pre")] +
                [(n, _f32p * 3) for n in ("ups_lrelu", "ups", "source_downs", "source_resblocks", "fusion")] +
                [("resblocks", _f32p * 9), ("post_resblocks", _f32p * 3)] +
                [(n, _f32p) for n in ("reflection_pad", "final_lrelu", "conv_post", "magnitude", "phase", "istft",
                                      "speech")])


def _declare(lib):
    if getattr(lib, "_hift_declared", False):
        return lib
    vp = ctypes.c_void_p
    lib.lx_hift_create.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
    lib.lx_hift_destroy.argtypes = [vp]
    lib.lx_hift_destroy.restype = None
    lib.lx_hift_last_error.argtypes = [vp]
    lib.lx_hift_last_error.restype = ctypes.c_char_p
    lib.lx_hift_load_gguf.argtypes = [vp, ctypes.c_char_p]
    lib.lx_hift_load_source.argtypes = [vp, ctypes.c_char_p]
    lib.lx_hift_vocode.argtypes = [vp, _f32p, ctypes.c_int, _f32p, _f32p, _f32p, ctypes.c_size_t,
                                   ctypes.POINTER(LxHiftDebug)]
    lib.lx_hift_vocode_device.argtypes = [vp, vp, ctypes.c_int, vp, vp]
    lib._hift_declared = True
    return lib


class HiftError(RuntimeError):
    pass


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def debug_shapes(T: int) -> dict:
    """Stage name -> shape of the captures (the reference's [C][len] layout)."""
    L_S = T * SAMPLES_PER_FRAME
    N = L_S // 4 + 1
    lens = (8 * T, 40 * T, 120 * T)
    ch = (256, 128, 64)
    s = {"f0": (T,), "sine_wavs": (L_S, HARMONICS), "sine_merge": (L_S,), "s_stft": (18, N),
         "conv_pre": (512, T)}
    cin = (512, 256, 128)
    lin = (T, 8 * T, 40 * T)
    for i in range(3):
        Lf = lens[i] + (1 if i == 2 else 0)
        s[f"ups{i}_lrelu"] = (cin[i], lin[i])
        s[f"ups{i}"] = (ch[i], lens[i])
        s[f"source_downs{i}"] = (ch[i], Lf)
        s[f"source_resblocks{i}"] = (ch[i], Lf)
        s[f"fusion{i}"] = (ch[i], Lf)
        for j in range(3):
            s[f"resblock{3 * i + j}"] = (ch[i], Lf)
        s[f"post_resblocks{i}"] = (ch[i], Lf)
    s.update({"reflection_pad": (64, N), "final_lrelu": (64, N), "conv_post": (18, N), "magnitude": (9, N),
              "phase": (9, N), "istft": (L_S,), "speech": (L_S,)})
    return s


class HiftVocoder:
    """Mirror of larynx::hift::HiftVocoder on one GPU (not thread-safe)."""

    def __init__(self, device: int = 0):
        self._lib = _declare(load_library())
        h = ctypes.c_void_p()
        rc = self._lib.lx_hift_create(int(device), ctypes.byref(h))
        if rc != LX_OK:
            raise HiftError(f"lx_hift_create(device={device}) failed: {ERRORS.get(rc, rc)} "
                            "(needs an sm_100 GPU; there is no CPU fallback)")
        self._h = h
        self.device = device

    def close(self):
        if getattr(self, "_h", None):
            self._lib.lx_hift_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def last_error(self) -> str:
        return self._lib.lx_hift_last_error(self._h).decode()

    def _check(self, rc: int, what: str) -> bool:
        if rc != LX_OK:
            print(f"hift: {what} failed: {ERRORS.get(rc, rc)}: {self.last_error}", file=sys.stderr)
            return False
        return True

    def load(self, gguf_path: str) -> bool:
        """HiftVocoder::load (hift.h:55)."""
        return self._check(self._lib.lx_hift_load_gguf(self._h, str(gguf_path).encode()), "load")

    def load_source(self, source_path: str) -> bool:
        """HiftVocoder::load_source (hift.h:63)."""
        return self._check(self._lib.lx_hift_load_source(self._h, str(source_path).encode()), "load_source")

    def vocode(self, mel, rand_ini=None, sine_waves=None, debug: Optional[dict] = None) -> Optional[np.ndarray]:
        """Both HiftVocoder::vocode overloads (hift.h:76-87): mel [80][T] (or
        (1, 80, T)) -> audio [T*480], or None on failure.  rand_ini [9] and
        sine_waves [T*480][9] are the explicit SineGen2 buffers (both or
        neither; neither = the loaded source).  A dict passed as `debug`
        receives every stage capture under the names of ``debug_shapes``."""
        mel = np.ascontiguousarray(np.asarray(mel, np.float32).reshape(80, -1))
        T = mel.shape[1]
        L_S = T * SAMPLES_PER_FRAME
        if (rand_ini is None) != (sine_waves is None):
            raise ValueError("rand_ini and sine_waves must both be given or both be None")
        ri = sw = None
        if rand_ini is not None:
            ri = np.ascontiguousarray(np.asarray(rand_ini, np.float32).reshape(HARMONICS))
            sw = np.ascontiguousarray(np.asarray(sine_waves, np.float32).reshape(-1, HARMONICS)[:L_S])
            if sw.shape[0] != L_S:
                print("hift: vocode failed: sine_waves shorter than T*480 rows", file=sys.stderr)
                return None
        audio = np.empty(L_S, np.float32)
        dbg_p = None
        bufs = {}
        if debug is not None:
            bufs = {k: np.empty(v, np.float32) for k, v in debug_shapes(T).items()}
            d = LxHiftDebug()
            for name in ("f0", "sine_wavs", "sine_merge", "s_stft", "conv_pre", "reflection_pad", "final_lrelu",
                         "conv_post", "magnitude", "phase", "istft", "speech"):
                setattr(d, name, _ptr(bufs[name]))
            for i in range(3):
                d.ups_lrelu[i] = _ptr(bufs[f"ups{i}_lrelu"])
                d.ups[i] = _ptr(bufs[f"ups{i}"])
                d.source_downs[i] = _ptr(bufs[f"source_downs{i}"])
                d.source_resblocks[i] = _ptr(bufs[f"source_resblocks{i}"])
                d.fusion[i] = _ptr(bufs[f"fusion{i}"])
                d.post_resblocks[i] = _ptr(bufs[f"post_resblocks{i}"])
            for j in range(9):
                d.resblocks[j] = _ptr(bufs[f"resblock{j}"])
            dbg_p = ctypes.byref(d)
        rc = self._lib.lx_hift_vocode(self._h, _ptr(mel), T, _ptr(ri) if ri is not None else None,
                                      _ptr(sw) if sw is not None else None, _ptr(audio), audio.size, dbg_p)
        if not self._check(rc, "vocode"):
            return None
        if debug is not None:
            debug.update(bufs)
        return audio

    def vocode_device(self, mel_ptr: int, T: int, audio_ptr: int, stream: int = 0) -> None:
        """Device form: mel [80][T] float32 at mel_ptr -> audio [T*480] at
        audio_ptr, enqueued on `stream` (the loaded source is used)."""
        rc = self._lib.lx_hift_vocode_device(self._h, ctypes.c_void_p(mel_ptr), int(T), ctypes.c_void_p(audio_ptr),
                                             ctypes.c_void_p(stream) if stream else None)
        if rc != LX_OK:
            raise HiftError(f"lx_hift_vocode_device: {ERRORS.get(rc, rc)}: {self.last_error}")


def conv_flops(T: int) -> int:
    """Algorithmic FLOPs (2 per multiply-add) of the float32 conv network for
    T mel frames: conv_pre, the upsample convs, source downsampling, the 12
    resblocks (6 convs each) and conv_post, at the layer's real channel counts."""
    f = 2 * 80 * 512 * 5 * T
    cin, L = 512, T
    for i, (r, k) in enumerate(zip((8, 5, 3), (16, 11, 7))):
        ch = 256 >> i
        L = L * r
        Lf = L + (1 if i == 2 else 0)
        f += 2 * cin * ch * k * L                         # ups
        f += 2 * 18 * ch * (30, 6, 1)[i] * Lf             # source_downs
        f += 6 * 2 * ch * ch * (7, 7, 11)[i] * Lf         # source resblock
        f += sum(6 * 2 * ch * ch * kk * Lf for kk in (3, 7, 11))
        cin = ch
    f += 2 * 64 * 18 * 7 * (120 * T + 1)                  # conv_post
    return f
