"""Python host side of the B200 Flow decoder: a ctypes binding of the C ABI
(include/larynx_flow.h) that mirrors larynx's ``FlowDecoder``
(include/larynx/flow/flow.h:39-82): ``load``, ``load_noise`` and ``infer``
keep the reference's names, argument meaning and bool-on-failure behaviour
(errors are also printed to stderr, as src/flow/flow.cpp:75-77 does).  The
batched CFM decode (``decode``), the device-pointer form (``decode_device``)
and the single estimator forward (``estimator``) extend it.

The CUDA library must be built (``make -C larynx_b200/csrc``); there is no CPU
fallback: loading fails loudly when ``liblarynx_flow.so`` is absent or the GPU
is not an sm_100 part.
"""

from __future__ import annotations

import ctypes
import os
import sys
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblarynx_flow.so")

LX_OK = 0
ERRORS = {1: "LX_ERR_ARG", 2: "LX_ERR_IO", 3: "LX_ERR_FORMAT", 4: "LX_ERR_SHAPE", 5: "LX_ERR_OOM",
          6: "LX_ERR_CUDA", 7: "LX_ERR_TIMEOUT", 8: "LX_ERR_STATE"}

# Symbols declared in include/larynx_flow.h
EXPORTS = ("lx_flow_create", "lx_flow_destroy", "lx_flow_last_error", "lx_flow_load_gguf", "lx_flow_load_noise",
           "lx_flow_infer", "lx_flow_decode", "lx_flow_decode_device", "lx_flow_estimator",
           "lx_flow_launch_count", "lx_flow_op", "lx_flow_op_gemm", "lx_flow_op_attention",
           "lx_flow_profile_decode", "lx_flow_op_attention_static", "lx_flow_infer_ex", "lx_flow_save_layout",
           "lx_flow_load_layout", "lx_flow_selftest_wait")

PRE_LOOKAHEAD = 3  # PreLookaheadLayer look-ahead tokens (cosyvoice3.yaml pre_lookahead_len)

KERNEL_CLASSES = ("in_proj", "conv_pos", "adaln", "qkv_gemm", "attention", "out_gemm", "ff1_gemm", "ff2_gemm",
                  "proj_out_gemm", "euler", "other")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


# lx_flow_debug: the stages of larynx::flow::FlowDebug (flow.h:15-34), in order
DEBUG_STAGES = ("spk", "token_embed", "prelookahead", "mu", "cond", "time_embed", "input_proj", "conv_pos",
                "input_embed", "blocks", "norm_out", "dphi")


class LxFlowDebug(ctypes.Structure):
    _fields_ = [(n, _f32p) for n in DEBUG_STAGES]


class LxFlowBatch(ctypes.Structure):
    _fields_ = [("n_utt", ctypes.c_int), ("lengths", _i32p), ("mu", ctypes.c_void_p), ("cond", ctypes.c_void_p),
                ("spks", ctypes.c_void_p), ("noise", ctypes.c_void_p), ("mel_out", ctypes.c_void_p),
                ("chunk", ctypes.c_int), ("n_steps", ctypes.c_int)]


_lib = None


def load_library(path: str = LIB_PATH):
    """Load liblarynx_flow.so and declare the C ABI.  Raises when absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `make -C {os.path.join(_HERE, 'csrc')}` "
                           "(the Flow decoder has no CPU fallback)")
    lib = ctypes.CDLL(path)
    vp = ctypes.c_void_p
    lib.lx_flow_create.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
    lib.lx_flow_destroy.argtypes = [vp]
    lib.lx_flow_destroy.restype = None
    lib.lx_flow_last_error.argtypes = [vp]
    lib.lx_flow_last_error.restype = ctypes.c_char_p
    lib.lx_flow_load_gguf.argtypes = [vp, ctypes.c_char_p]
    lib.lx_flow_load_noise.argtypes = [vp, ctypes.c_char_p]
    lib.lx_flow_save_layout.argtypes = [vp, ctypes.c_char_p]
    lib.lx_flow_load_layout.argtypes = [vp, ctypes.c_char_p]
    lib.lx_flow_infer.argtypes = [vp, _i32p, ctypes.c_int, _i32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p, _f32p,
                                  _f32p, ctypes.c_size_t, ctypes.POINTER(LxFlowDebug)]
    lib.lx_flow_infer_ex.argtypes = [vp, _i32p, ctypes.c_int, _i32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p, _f32p,
                                     ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_size_t, ctypes.POINTER(LxFlowDebug)]
    lib.lx_flow_decode.argtypes = [vp, ctypes.POINTER(LxFlowBatch)]
    lib.lx_flow_decode_device.argtypes = [vp, ctypes.POINTER(LxFlowBatch), vp]
    lib.lx_flow_estimator.argtypes = [vp, ctypes.c_int, _i32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float,
                                      ctypes.c_int, _f32p, _f32p, _f32p, ctypes.c_int, _f32p]
    lib.lx_flow_launch_count.argtypes = [vp]
    lib.lx_flow_launch_count.restype = ctypes.c_uint64
    lib.lx_flow_op.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp, _f32p, _f32p, _f32p, _i32p, vp]
    lib.lx_flow_profile_decode.argtypes = [vp, ctypes.POINTER(LxFlowBatch), vp, ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    lib.lx_flow_profile_decode.restype = ctypes.c_int
    lib.lx_flow_op_gemm.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp, vp]
    lib.lx_flow_op_attention.argtypes = [ctypes.c_int, _i32p, vp, vp, vp, vp, ctypes.c_int, vp]
    lib.lx_flow_op_attention_static.argtypes = [ctypes.c_int, _i32p, vp, vp, vp, vp, ctypes.c_int, vp]
    lib.lx_flow_selftest_wait.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.POINTER(ctypes.c_int), vp]
    for name in ("lx_flow_selftest_wait", "lx_flow_op_gemm", "lx_flow_op_attention", "lx_flow_op_attention_static", "lx_flow_infer_ex",
                 "lx_flow_save_layout", "lx_flow_load_layout", "lx_flow_create", "lx_flow_load_gguf", "lx_flow_load_noise", "lx_flow_infer", "lx_flow_decode",
                 "lx_flow_decode_device", "lx_flow_estimator", "lx_flow_op"):
        getattr(lib, name).restype = ctypes.c_int
    _lib = lib
    return lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(_f32p)


class FlowError(RuntimeError):
    pass


class FlowDecoder:
    """Mirror of larynx::flow::FlowDecoder on one GPU (not thread-safe)."""

    def __init__(self, device: int = 0):
        self._lib = load_library()
        h = ctypes.c_void_p()
        rc = self._lib.lx_flow_create(int(device), ctypes.byref(h))
        if rc != LX_OK:
            raise FlowError(f"lx_flow_create(device={device}) failed: {ERRORS.get(rc, rc)} "
                            "(needs an sm_100 GPU; there is no CPU fallback)")
        self._h = h
        self.device = device

    def close(self):
        if getattr(self, "_h", None):
            self._lib.lx_flow_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def last_error(self) -> str:
        return self._lib.lx_flow_last_error(self._h).decode()

    @property
    def launch_count(self) -> int:
        return int(self._lib.lx_flow_launch_count(self._h))

    def _check(self, rc: int, what: str) -> bool:
        if rc != LX_OK:
            print(f"flow: {what} failed: {ERRORS.get(rc, rc)}: {self.last_error}", file=sys.stderr)
            return False
        return True

    def _raise(self, rc: int, what: str):
        if rc != LX_OK:
            raise FlowError(f"{what}: {ERRORS.get(rc, rc)}: {self.last_error}")

    # --- reference interface -------------------------------------------
    def load(self, gguf_path: str) -> bool:
        """FlowDecoder::load (flow.h:48)."""
        return self._check(self._lib.lx_flow_load_gguf(self._h, gguf_path.encode()), "load")

    def save_layout(self, path: str) -> bool:
        """Write the loaded model's device layout (pre-laid-out weight cache)."""
        return self._check(self._lib.lx_flow_save_layout(self._h, path.encode()), "save_layout")

    def load_layout(self, path: str) -> bool:
        """Load a file written by save_layout instead of a flow.gguf."""
        return self._check(self._lib.lx_flow_load_layout(self._h, path.encode()), "load_layout")

    def load_noise(self, noise_path: str) -> bool:
        """FlowDecoder::load_noise (flow.h:55)."""
        return self._check(self._lib.lx_flow_load_noise(self._h, noise_path.encode()), "load_noise")

    def infer(self, prompt_tokens: Sequence[int], tokens: Sequence[int], prompt_feat, spk_embedding,
              noise_z=None, debug: Optional[dict] = None, finalize: bool = True,
              chunk: int = 0) -> Optional[np.ndarray]:
        """FlowDecoder::infer (flow.h:61-77): token -> mel [80, MEL_T - mel_len1],
        or None on failure.  noise_z [80, >= MEL_T] (its first MEL_T columns)
        or None (slice of the loaded bank).  ``debug`` (a dict) receives the
        step-1 stage captures.  ``finalize=False`` is the reference's streaming
        call (flow_reference.py:546-548): the last 3 tokens are PreLookahead
        context and MEL_T = 2 * (tokens - 3).  ``chunk`` > 0 applies the
        block-causal chunk mask (upstream CosyVoice3's streaming attention)."""
        pt = np.ascontiguousarray(np.asarray(prompt_tokens, dtype=np.int32).reshape(-1))
        tk = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        pf = _f32(prompt_feat).reshape(-1, 80)
        spk = _f32(spk_embedding).reshape(-1)
        T = 2 * (pt.size + tk.size - (0 if finalize else PRE_LOOKAHEAD))
        nz = None
        if noise_z is not None:
            z = np.asarray(noise_z, np.float32).reshape(80, -1)
            if z.shape[1] < T:
                raise ValueError(f"noise_z has {z.shape[1]} frames, {T} needed")
            nz = _f32(z[:, :T])
        out = np.empty((80, max(T - pf.shape[0], 0)), np.float32)
        dbg = None
        bufs = {}
        if debug is not None:
            n_tok = pt.size + tk.size
            n_pre = n_tok - (0 if finalize else PRE_LOOKAHEAD)
            shapes = {"spk": (80,), "token_embed": (n_tok, 80), "prelookahead": (n_pre, 80), "mu": (80, T),
                      "cond": (80, T), "time_embed": (2, 1024), "input_proj": (2, T, 1024),
                      "conv_pos": (2, T, 1024), "input_embed": (2, T, 1024), "blocks": (22, 2, T, 1024),
                      "norm_out": (2, T, 1024), "dphi": (2, 80, T)}
            bufs = {k: np.empty(v, np.float32) for k, v in shapes.items()}
            dbg = LxFlowDebug(**{k: _ptr(v) for k, v in bufs.items()})
        rc = self._lib.lx_flow_infer_ex(self._h, pt.ctypes.data_as(_i32p), pt.size, tk.ctypes.data_as(_i32p),
                                        tk.size, _ptr(pf), pf.shape[0], _ptr(spk), _ptr(nz), int(bool(finalize)),
                                        int(chunk), _ptr(out), out.size,
                                        ctypes.byref(dbg) if dbg is not None else None)
        if not self._check(rc, "infer"):
            return None
        if debug is not None:
            debug.update(bufs)
        return out

    # --- extensions ----------------------------------------------------
    def decode(self, lengths: Sequence[int], mu, cond, spks, noise=None, chunk: int = 0,
               n_steps: int = 0, out: Optional[np.ndarray] = None) -> np.ndarray:
        """Batched 10-step CFG decode.  mu/cond/noise: concatenation of the
        utterances' [80, T_u] blocks (flat or a list of arrays); spks [U, 80].
        Returns the flat concatenation of the final [80, T_u] blocks (written
        into ``out`` when given: float32, contiguous, sum(T_u) * 80)."""
        L = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
        cat = lambda a: _f32(np.concatenate([np.asarray(x, np.float32).reshape(-1) for x in a])
                             if isinstance(a, (list, tuple)) else np.asarray(a, np.float32).reshape(-1))
        mu_, cond_ = cat(mu), cat(cond)
        nz = None if noise is None else cat(noise)
        sp = _f32(spks).reshape(-1)
        n = int(L.sum()) * 80
        if out is None:
            out = np.empty(n, np.float32)
        elif out.dtype != np.float32 or out.size != n or not out.flags["C_CONTIGUOUS"]:
            raise ValueError("out must be a contiguous float32 array of sum(lengths) * 80 elements")
        if mu_.size != n or cond_.size != n or (nz is not None and nz.size != n) or sp.size != 80 * L.size:
            raise ValueError("input sizes do not match the lengths")
        b = LxFlowBatch(int(L.size), L.ctypes.data_as(_i32p), mu_.ctypes.data, cond_.ctypes.data, sp.ctypes.data,
                        None if nz is None else nz.ctypes.data, out.ctypes.data, int(chunk), int(n_steps))
        self._raise(self._lib.lx_flow_decode(self._h, ctypes.byref(b)), "decode")
        return out

    def decode_device(self, lengths: np.ndarray, mu_ptr: int, cond_ptr: int, spks_ptr: int, noise_ptr: int,
                      out_ptr: int, chunk: int = 0, stream: int = 0, n_steps: int = 0) -> None:
        """Device-pointer decode enqueued on ``stream`` (no synchronisation).
        n_steps 0 runs the full 10-step schedule, 1..10 its first n steps."""
        L = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
        self._dev_lengths = L  # keep alive for the call
        b = LxFlowBatch(int(L.size), L.ctypes.data_as(_i32p), mu_ptr, cond_ptr, spks_ptr, noise_ptr, out_ptr,
                        int(chunk), int(n_steps))
        self._raise(self._lib.lx_flow_decode_device(self._h, ctypes.byref(b), ctypes.c_void_p(stream or None)),
                    "decode_device")

    def profile_decode(self, lengths, mu_ptr: int, cond_ptr: int, spks_ptr: int, noise_ptr: int, out_ptr: int,
                       chunk: int = 0, stream: int = 0) -> dict:
        """Device-pointer decode without graphs, every kernel bracketed by CUDA
        events; returns {class: (total_ms, launches)}."""
        L = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
        b = LxFlowBatch(int(L.size), L.ctypes.data_as(_i32p), mu_ptr, cond_ptr, spks_ptr, noise_ptr, out_ptr,
                        int(chunk), 0)
        n = len(KERNEL_CLASSES)
        ms = (ctypes.c_double * n)()
        cnt = (ctypes.c_int * n)()
        self._raise(self._lib.lx_flow_profile_decode(self._h, ctypes.byref(b), ctypes.c_void_p(stream or None), ms,
                                                     cnt, n), "profile_decode")
        return {k: (ms[i], cnt[i]) for i, k in enumerate(KERNEL_CLASSES)}

    def estimator(self, lengths: Sequence[int], x, mu, cond, spks, t: float, chunk: int = 0,
                  capture_block: Optional[int] = None, want_input_embed=False, want_norm_out=False):
        """One DiT forward over independent sequences (flat [80, T_s] blocks).
        Returns (dphi_flat, captures)."""
        L = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
        tot = int(L.sum())
        x_, mu_, cond_ = _f32(x).reshape(-1), _f32(mu).reshape(-1), _f32(cond).reshape(-1)
        sp = _f32(spks).reshape(-1)
        dphi = np.empty(tot * 80, np.float32)
        ie = np.empty((tot, 1024), np.float32) if want_input_embed else None
        bo = np.empty((tot, 1024), np.float32) if capture_block is not None else None
        no = np.empty((tot, 1024), np.float32) if want_norm_out else None
        rc = self._lib.lx_flow_estimator(self._h, int(L.size), L.ctypes.data_as(_i32p), _ptr(x_), _ptr(mu_),
                                         _ptr(cond_), _ptr(sp), float(t), int(chunk), _ptr(dphi), _ptr(ie), _ptr(bo),
                                         -1 if capture_block is None else int(capture_block), _ptr(no))
        self._raise(rc, "estimator")
        return dphi, {"input_embed": ie, "block": bo, "norm_out": no}


def op(op_id: int, in_bf16: bool, rows: int, x_ptr: int, y_ptr: int, shift_ptr=0, scale_ptr=0, gate_ptr=0,
       pos_ptr=0, stream: int = 0) -> None:
    """Standalone fused op on device pointers (0 AdaLN-mod, 1 gate-residual,
    2 partial rotary, 3 GELU-tanh)."""
    lib = load_library()
    c = lambda p, t=_f32p: ctypes.cast(ctypes.c_void_p(p), t) if p else None
    rc = lib.lx_flow_op(op_id, int(in_bf16), rows, ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), c(shift_ptr),
                        c(scale_ptr), c(gate_ptr), c(pos_ptr, _i32p), ctypes.c_void_p(stream or None))
    if rc != LX_OK:
        raise FlowError(f"lx_flow_op({op_id}) failed: {ERRORS.get(rc, rc)}")


def op_gemm(M: int, N: int, K: int, a_ptr: int, b_ptr: int, bias_ptr: int, c_ptr: int, stream: int = 0) -> None:
    """C[M,N] fp32 = A[M,K] @ B[N,K]^T (+bias) on the tcgen05 GEMM (device pointers)."""
    lib = load_library()
    v = lambda p: ctypes.c_void_p(p) if p else None
    rc = lib.lx_flow_op_gemm(M, N, K, v(a_ptr), v(b_ptr), v(bias_ptr), v(c_ptr), v(stream))
    if rc != LX_OK:
        raise FlowError(f"lx_flow_op_gemm failed: {ERRORS.get(rc, rc)}")


def op_attention(lengths, q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, chunk: int = 0, stream: int = 0) -> None:
    """Flash attention over packed bf16 [R,1024] rows (device pointers)."""
    lib = load_library()
    L = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
    v = lambda p: ctypes.c_void_p(p) if p else None
    rc = lib.lx_flow_op_attention(int(L.size), L.ctypes.data_as(_i32p), v(q_ptr), v(k_ptr), v(v_ptr), v(out_ptr),
                                  int(chunk), v(stream))
    if rc != LX_OK:
        raise FlowError(f"lx_flow_op_attention failed: {ERRORS.get(rc, rc)}")


def op_attention_static(lengths, q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, chunk: int = 0,
                        stream: int = 0) -> None:
    """``op_attention`` for callers that may not allocate device memory: the
    scratch is fixed static device storage (packed rows <= 4096).  Calls that overlap in time on one device race on that storage."""
    lib = load_library()
    L = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
    v = lambda p: ctypes.c_void_p(p) if p else None
    rc = lib.lx_flow_op_attention_static(int(L.size), L.ctypes.data_as(_i32p), v(q_ptr), v(k_ptr), v(v_ptr),
                                         v(out_ptr), int(chunk), v(stream))
    if rc != LX_OK:
        raise FlowError(f"lx_flow_op_attention_static failed: {ERRORS.get(rc, rc)}")


def selftest_wait(producer_arrives: bool, limit_ms: float, stream: int = 0):
    """Run the bounded-wait self test (lx_flow_selftest_wait): returns
    (status, device error code).  status is LX_OK when the producer arrived
    and 7 (LX_ERR_TIMEOUT) when the wait ran out after ``limit_ms``."""
    lib = load_library()
    code = ctypes.c_int(-1)
    rc = lib.lx_flow_selftest_wait(int(bool(producer_arrives)), float(limit_ms), ctypes.byref(code),
                                   ctypes.c_void_p(stream or None))
    return rc, code.value
