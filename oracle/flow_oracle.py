"""CPU oracle for the Flow decoder hot path (TEST INFRASTRUCTURE ONLY).

This module is the parity checker for the CUDA implementation in
``larynx_b200``.  It restates, in plain numpy (float32 by default, float64 on
request), the reference's own ground-truth Flow model:

  * ``tests/flow_reference.py`` of hardenedlinux/larynx (the PyTorch statement
    of CosyVoice3's ``CausalMaskedDiffWithDiT`` + DiT estimator + CFM), and
  * the GGML graph of ``src/flow/{dit,ops,flow,flow_matching,prelookahead}.cpp``
    for layouts, the Euler/CFG order and the chunk order of the modulation.

Every function cites the reference file:line it follows.  Parity of this
restatement is pinned against the reference itself: ``tests/golden/make_golden.py``
imports the reference's ``flow_reference.py`` (in the build container only),
runs it on seeded synthetic weights and stores stage-by-stage golden vectors
under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module
against them.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker / CPU baseline.  The
product path (``larynx_b200``) never calls it.
"""

from __future__ import annotations

import math
import zlib
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

# ---------------------------------------------------------------------------
# Architecture constants: src/flow/internal.h:18-41, flow_reference.py:577-590
# ---------------------------------------------------------------------------
MEL_DIM = 80
SPK_EMBED_DIM = 192
VOCAB = 6561
DIM = 1024
HEADS = 16
HEAD_DIM = 64
ROT_DIM = 64
FF_INNER = 2048
DEPTH = 22
PRE_LOOKAHEAD = 3
TOKEN_MEL_RATIO = 2
N_TIMESTEPS = 10
CFG_RATE = 0.7
CONV_POS_KERNEL = 31
CONV_POS_GROUPS = 16
LN_EPS = 1e-6
ROPE_BASE = 10000.0
NOISE_MAX_FRAMES = 50 * 300

EST = "decoder.estimator."


# ---------------------------------------------------------------------------
# Parameter inventory (names and torch shapes of the 330 state_dict entries).
# Names: src/flow/gguf.cpp:46-90; shapes: src/flow/internal.h:50-93 (ne
# reversed), flow_reference.py:577-590.
# ---------------------------------------------------------------------------
def param_specs() -> List[Tuple[str, Tuple[int, ...]]]:
    s: List[Tuple[str, Tuple[int, ...]]] = [
        ("input_embedding.weight", (VOCAB, MEL_DIM)),
        ("spk_embed_affine_layer.weight", (MEL_DIM, SPK_EMBED_DIM)),
        ("spk_embed_affine_layer.bias", (MEL_DIM,)),
        ("pre_lookahead_layer.conv1.weight", (DIM, MEL_DIM, PRE_LOOKAHEAD + 1)),
        ("pre_lookahead_layer.conv1.bias", (DIM,)),
        ("pre_lookahead_layer.conv2.weight", (MEL_DIM, DIM, 3)),
        ("pre_lookahead_layer.conv2.bias", (MEL_DIM,)),
        (EST + "time_embed.time_mlp.0.weight", (DIM, 256)),
        (EST + "time_embed.time_mlp.0.bias", (DIM,)),
        (EST + "time_embed.time_mlp.2.weight", (DIM, DIM)),
        (EST + "time_embed.time_mlp.2.bias", (DIM,)),
        (EST + "input_embed.proj.weight", (DIM, 4 * MEL_DIM)),
        (EST + "input_embed.proj.bias", (DIM,)),
        (EST + "input_embed.conv_pos_embed.conv1.0.weight", (DIM, DIM // CONV_POS_GROUPS, CONV_POS_KERNEL)),
        (EST + "input_embed.conv_pos_embed.conv1.0.bias", (DIM,)),
        (EST + "input_embed.conv_pos_embed.conv2.0.weight", (DIM, DIM // CONV_POS_GROUPS, CONV_POS_KERNEL)),
        (EST + "input_embed.conv_pos_embed.conv2.0.bias", (DIM,)),
        (EST + "rotary_embed.inv_freq", (ROT_DIM // 2,)),
    ]
    for i in range(DEPTH):
        b = f"{EST}transformer_blocks.{i}."
        s += [
            (b + "attn_norm.linear.weight", (6 * DIM, DIM)),
            (b + "attn_norm.linear.bias", (6 * DIM,)),
            (b + "attn.to_q.weight", (DIM, DIM)),
            (b + "attn.to_q.bias", (DIM,)),
            (b + "attn.to_k.weight", (DIM, DIM)),
            (b + "attn.to_k.bias", (DIM,)),
            (b + "attn.to_v.weight", (DIM, DIM)),
            (b + "attn.to_v.bias", (DIM,)),
            (b + "attn.to_out.0.weight", (DIM, DIM)),
            (b + "attn.to_out.0.bias", (DIM,)),
            (b + "ff.ff.0.0.weight", (FF_INNER, DIM)),
            (b + "ff.ff.0.0.bias", (FF_INNER,)),
            (b + "ff.ff.2.weight", (DIM, FF_INNER)),
            (b + "ff.ff.2.bias", (DIM,)),
        ]
    s += [
        (EST + "norm_out.linear.weight", (2 * DIM, DIM)),
        (EST + "norm_out.linear.bias", (2 * DIM,)),
        (EST + "proj_out.weight", (MEL_DIM, DIM)),
        (EST + "proj_out.bias", (MEL_DIM,)),
    ]
    return s


def rotary_inv_freq() -> np.ndarray:
    """inv_freq = 1 / base^(arange(0, 64, 2)/64), float32 ops in torch order
    (flow_reference.py:78-80)."""
    ar = np.arange(0, ROT_DIM, 2).astype(np.float32) / np.float32(ROT_DIM)
    return (np.float32(1.0) / np.power(np.float32(ROPE_BASE), ar).astype(np.float32)).astype(np.float32)


def synth_tensor(name: str, shape: Sequence[int], seed: int = 0, std: float = 0.02) -> np.ndarray:
    """One synthetic weight: N(0, std) from a per-name PCG64 stream, so any
    subset can be regenerated independently of order.  ``inv_freq`` is a
    derived buffer, not a weight: it keeps its formula value."""
    if name.endswith("rotary_embed.inv_freq"):
        return rotary_inv_freq()
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    return (rng.standard_normal(tuple(shape), dtype=np.float32) * np.float32(std)).astype(np.float32)


def synth_weights(seed: int = 0, std: float = 0.02) -> Dict[str, np.ndarray]:
    """All 330 state_dict tensors with synthetic N(0, std) values (BASELINE
    config 0 weight init: seed 0, std 0.02)."""
    return {n: synth_tensor(n, sh, seed, std) for n, sh in param_specs()}


# ---------------------------------------------------------------------------
# Elementwise pieces
# ---------------------------------------------------------------------------
def silu(x):
    """nn.SiLU (flow_reference.py:172, 298)."""
    return x / (1.0 + np.exp(-x))


def gelu_tanh(x):
    """nn.GELU(approximate='tanh') (flow_reference.py:202, 282); same constants
    as src/flow/ops.cpp:73-83."""
    c1 = x.dtype.type(0.7978845608028654)
    c0 = x.dtype.type(0.044715)
    return x.dtype.type(0.5) * x * (x.dtype.type(1.0) + np.tanh(c1 * (x + c0 * x * x * x)))


def mish(x):
    """nn.Mish = x * tanh(softplus(x)) (flow_reference.py:147, 151;
    src/flow/ops.cpp:69-71).  softplus uses torch's threshold of 20."""
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    return x * np.tanh(sp)


def layer_norm(x, eps=LN_EPS):
    """LayerNorm without affine, biased variance (flow_reference.py:174, 188,
    281; src/flow/ops.cpp:94-104 ggml_norm)."""
    mu = x.mean(axis=-1, keepdims=True)
    xc = x - mu
    var = (xc * xc).mean(axis=-1, keepdims=True)
    return xc / np.sqrt(var + x.dtype.type(eps))


def linear(x, w, b=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    return y


# ---------------------------------------------------------------------------
# Timestep embedding: flow_reference.py:125-137, 294-304;
# src/flow/flow_matching.cpp:10-42
# ---------------------------------------------------------------------------
def sinus_embed(t: np.ndarray, dim: int = 256, scale: float = 1000.0) -> np.ndarray:
    t = np.asarray(t, dtype=np.float32).reshape(-1)
    half = dim // 2
    e = math.log(10000) / (half - 1)
    freqs = np.exp(np.arange(half, dtype=np.float32) * np.float32(-e)).astype(np.float32)
    ang = np.float32(scale) * t[:, None] * freqs[None, :]
    return np.concatenate([np.sin(ang), np.cos(ang)], axis=-1).astype(np.float32)


def time_embed(W, t, dtype=np.float32) -> np.ndarray:
    h = sinus_embed(t).astype(dtype)
    h = linear(h, W[EST + "time_embed.time_mlp.0.weight"].astype(dtype), W[EST + "time_embed.time_mlp.0.bias"].astype(dtype))
    h = silu(h)
    return linear(h, W[EST + "time_embed.time_mlp.2.weight"].astype(dtype), W[EST + "time_embed.time_mlp.2.bias"].astype(dtype))


def adaln_chunks(W, i: int, temb, dtype=np.float32):
    """AdaLayerNormZero emb chunks, in the order shift_msa, scale_msa,
    gate_msa, shift_mlp, scale_mlp, gate_mlp (flow_reference.py:176-180;
    src/flow/dit.cpp:56-62)."""
    b = f"{EST}transformer_blocks.{i}.attn_norm.linear."
    emb = linear(silu(temb), W[b + "weight"].astype(dtype), W[b + "bias"].astype(dtype))
    return np.split(emb, 6, axis=-1)


def final_chunks(W, temb, dtype=np.float32):
    """AdaLayerNormZero_Final emb chunks in the order scale, shift
    (flow_reference.py:190-193; src/flow/dit.cpp:133-136)."""
    emb = linear(silu(temb), W[EST + "norm_out.linear.weight"].astype(dtype), W[EST + "norm_out.linear.bias"].astype(dtype))
    return np.split(emb, 2, axis=-1)


def ada_ln(x, scale, shift):
    """norm(x) * (1 + scale) + shift, modulation broadcast over the sequence
    (flow_reference.py:179, 288, 193; src/flow/ops.cpp:94-104).
    x: [B, T, D]; scale/shift: [B, D]."""
    return layer_norm(x) * (x.dtype.type(1.0) + scale[:, None, :]) + shift[:, None, :]


# ---------------------------------------------------------------------------
# Partial rotary: flow_reference.py:52-106, 217-221; src/flow/ops.cpp:85-92
# ---------------------------------------------------------------------------
def rotary_cos_sin(T: int, dtype=np.float32):
    """freqs[p, 2i] = freqs[p, 2i+1] = p * inv_freq[i] (GPT-J interleaved pairs,
    flow_reference.py:93-98); positions 0..T-1 (src/flow/flow.cpp:226-229)."""
    pos = np.arange(T, dtype=np.float32)
    f = (pos[:, None] * rotary_inv_freq()[None, :]).astype(np.float32)  # [T, 32]
    f = np.repeat(f, 2, axis=-1)                                          # [T, 64]
    return np.cos(f).astype(dtype), np.sin(f).astype(dtype)


def rotate_half(x):
    """(x0, x1) -> (-x1, x0) over adjacent pairs (flow_reference.py:52-56)."""
    x2 = x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2)
    out = np.stack((-x2[..., 1], x2[..., 0]), axis=-1)
    return out.reshape(x.shape)


def apply_rotary_partial(x, cos, sin):
    """Rotate only the first 64 channels of the full 1024-wide projection
    (flow_reference.py:59-71 applied before the head split at :220-221).
    x: [B, T, D]; cos/sin: [T, 64]."""
    r, u = x[..., :ROT_DIM], x[..., ROT_DIM:]
    r = r * cos + rotate_half(r) * sin
    return np.concatenate([r, u], axis=-1)


# ---------------------------------------------------------------------------
# Attention: flow_reference.py:210-249; src/flow/dit.cpp:34-51
# ---------------------------------------------------------------------------
def sdpa(q, k, v, mask):
    """softmax(q k^T / sqrt(64) + mask) v per (batch, head).
    q/k/v: [B, T, D]; mask: bool [B, T(query), T(key)] (True = attend) or None."""
    B, T, _ = q.shape
    scale = q.dtype.type(1.0 / math.sqrt(HEAD_DIM))
    out = np.empty_like(q)
    for b in range(B):
        for h in range(HEADS):
            sl = slice(h * HEAD_DIM, (h + 1) * HEAD_DIM)
            s = (q[b, :, sl] @ k[b, :, sl].T) * scale
            if mask is not None:
                s = np.where(mask[b], s, -np.inf)
            m = s.max(axis=-1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            p = np.exp(s - m)
            p = p / p.sum(axis=-1, keepdims=True)
            out[b, :, sl] = p @ v[b, :, sl]
    return out


def attention(W, i, x, mask, cos, sin, capture=None):
    b = f"{EST}transformer_blocks.{i}.attn."
    q = linear(x, W[b + "to_q.weight"], W[b + "to_q.bias"])
    k = linear(x, W[b + "to_k.weight"], W[b + "to_k.bias"])
    v = linear(x, W[b + "to_v.weight"], W[b + "to_v.bias"])
    q = apply_rotary_partial(q, cos, sin)
    k = apply_rotary_partial(k, cos, sin)
    o = sdpa(q, k, v, mask)
    if capture is not None:
        capture.update(q=q, k=k, v=v, attn_core=o)
    o = linear(o, W[b + "to_out.0.weight"], W[b + "to_out.0.bias"])
    if mask is not None:
        # padded query rows are zeroed after to_out (flow_reference.py:243-248:
        # the row mask is the last query row's key mask, mask[:, 0, -1]).
        o = np.where(mask[:, -1, :][:, :, None], o, 0.0).astype(o.dtype)
    return o


def feed_forward(W, i, x):
    """Linear 1024->2048, GELU-tanh, Linear 2048->1024 (flow_reference.py:197-207)."""
    b = f"{EST}transformer_blocks.{i}.ff.ff."
    h = gelu_tanh(linear(x, W[b + "0.0.weight"], W[b + "0.0.bias"]))
    return linear(h, W[b + "2.weight"], W[b + "2.bias"])


def dit_block(W, i, x, temb, mask, cos, sin, capture=None):
    """DiTBlock.forward (flow_reference.py:284-291; src/flow/dit.cpp:53-79)."""
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = adaln_chunks(W, i, temb, x.dtype)
    norm = ada_ln(x, scale_msa, shift_msa)
    a = attention(W, i, norm, mask, cos, sin, capture)
    x = x + gate_msa[:, None, :] * a
    ffn = ada_ln(x, scale_mlp, shift_mlp)
    x = x + gate_mlp[:, None, :] * feed_forward(W, i, ffn)
    return x


# ---------------------------------------------------------------------------
# Input embedding + causal grouped conv position embedding:
# flow_reference.py:140-166, 310-330; src/flow/dit.cpp:104-123, ops.cpp:45-71
# ---------------------------------------------------------------------------
def grouped_causal_conv(x, w, b):
    """Left pad 30, Conv1d(1024, 1024, k=31, groups=16).  x: [B, T, D] ->
    [B, T, D].  w: [1024, 64, 31]."""
    B, T, D = x.shape
    G = CONV_POS_GROUPS
    cg = D // G
    K = CONV_POS_KERNEL
    xp = np.concatenate([np.zeros((B, K - 1, D), x.dtype), x], axis=1)   # [B, T+30, D]
    out = np.empty((B, T, D), x.dtype)
    for g in range(G):
        xs = xp[:, :, g * cg:(g + 1) * cg]                                  # [B, T+30, 64]
        # im2col over taps: cols[b, t, k, i] = xs[b, t + k, i]
        cols = np.stack([xs[:, k:k + T, :] for k in range(K)], axis=2)      # [B, T, 31, 64]
        wg = w[g * cg:(g + 1) * cg]                                         # [64(o), 64(i), 31(k)]
        wk = np.transpose(wg, (0, 2, 1)).reshape(cg, K * cg)               # [o, k*64+i]
        out[:, :, g * cg:(g + 1) * cg] = cols.reshape(B, T, K * cg) @ wk.T + b[g * cg:(g + 1) * cg]
    return out


def conv_pos_embed(W, x):
    p = EST + "input_embed.conv_pos_embed."
    h = mish(grouped_causal_conv(x, W[p + "conv1.0.weight"].astype(x.dtype), W[p + "conv1.0.bias"].astype(x.dtype)))
    return mish(grouped_causal_conv(h, W[p + "conv2.0.weight"].astype(x.dtype), W[p + "conv2.0.bias"].astype(x.dtype)))


def input_embed(W, x, cond, mu, spks, capture=None):
    """proj(cat[x, cond, mu, spks]) + conv_pos (flow_reference.py:318-330;
    concat order src/flow/dit.cpp:109).  x/cond/mu: [B, T, 80]; spks: [B, 80]."""
    B, T, _ = x.shape
    cat = np.concatenate([x, cond, mu, np.broadcast_to(spks[:, None, :], (B, T, MEL_DIM))], axis=-1)
    xe = linear(cat, W[EST + "input_embed.proj.weight"].astype(x.dtype), W[EST + "input_embed.proj.bias"].astype(x.dtype))
    pos = conv_pos_embed(W, xe)
    if capture is not None:
        capture["input_proj"] = xe
        capture["conv_pos"] = pos
    return pos + xe


# ---------------------------------------------------------------------------
# Masks: flow_reference.py:112-119 (make_pad_mask), :375-380
# ---------------------------------------------------------------------------
def key_padding_mask(lengths: Sequence[int], T: int) -> np.ndarray:
    """[B, T(query), T(key)]: key j visible iff j < len (non-streaming mask
    repeated over queries, flow_reference.py:380)."""
    lengths = np.asarray(lengths)
    kv = np.arange(T)[None, :] < lengths[:, None]
    return np.broadcast_to(kv[:, None, :], (len(lengths), T, T)).copy()


def block_causal_mask(lengths: Sequence[int], T: int, chunk: int) -> np.ndarray:
    """Block-causal chunk mask: query i sees key j iff floor(j/chunk) <=
    floor(i/chunk) and j < len.  The reference has no streaming path
    (docs/FLOW.md:470-472); this is the documented extension, passed to the
    estimator through its streaming [B, T, T] mask input
    (flow_reference.py:375-376)."""
    lengths = np.asarray(lengths)
    ci = np.arange(T) // chunk
    vis = ci[None, :] <= ci[:, None]                              # [T(q), T(k)]
    kv = np.arange(T)[None, :] < lengths[:, None]                 # [B, T(k)]
    return vis[None, :, :] & kv[:, None, :]


# ---------------------------------------------------------------------------
# DiT forward: flow_reference.py:355-400; src/flow/dit.cpp:83-145
# ---------------------------------------------------------------------------
def dit_forward(W, x, mu, t, spks, cond, mask=None, capture=None):
    """x/mu/cond: [B, 80, T] (PyTorch (B, C, T)); t: [B]; spks: [B, 80];
    mask: bool [B, T, T] or None (= all visible).  Returns dphi [B, 80, T]."""
    dtype = x.dtype
    xt = np.ascontiguousarray(np.transpose(x, (0, 2, 1)))
    mut = np.ascontiguousarray(np.transpose(mu, (0, 2, 1)))
    condt = np.ascontiguousarray(np.transpose(cond, (0, 2, 1)))
    B, T, _ = xt.shape
    temb = time_embed(W, np.asarray(t, np.float32).reshape(-1), dtype)
    if temb.shape[0] == 1 and B > 1:
        temb = np.repeat(temb, B, axis=0)
    if capture is not None:
        capture["time_embed"] = temb
    h = input_embed(W, xt, condt, mut, spks.astype(dtype), capture)
    if capture is not None:
        capture["input_embed"] = h
        capture["blocks"] = []
    cos, sin = rotary_cos_sin(T, dtype)
    for i in range(DEPTH):
        h = dit_block(W, i, h, temb, mask, cos, sin)
        if capture is not None:
            capture["blocks"].append(h)
    scale, shift = final_chunks(W, temb, dtype)
    h = ada_ln(h, scale, shift)
    if capture is not None:
        capture["norm_out"] = h
    out = linear(h, W[EST + "proj_out.weight"].astype(dtype), W[EST + "proj_out.bias"].astype(dtype))
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1)))


# ---------------------------------------------------------------------------
# CFM Euler solver with CFG: flow_reference.py:468-501; src/flow/flow.cpp:202-274
# ---------------------------------------------------------------------------
def t_span_cosine(n: int = N_TIMESTEPS) -> np.ndarray:
    """t_span = 1 - cos(linspace(0, 1, n+1) * pi/2), float32
    (flow_reference.py:471-473; src/flow/flow.cpp:202-207)."""
    ls = np.linspace(0, 1, n + 1, dtype=np.float32)
    return (np.float32(1.0) - np.cos(ls * np.float32(0.5 * math.pi))).astype(np.float32)


def euler_schedule(n: int = N_TIMESTEPS) -> List[Tuple[float, float]]:
    """The (t, dt) pair used at each step, accumulated in float32 exactly as
    solve_euler does (t += dt; dt = t_span[step+1] - t; flow_reference.py:477-500)."""
    ts = t_span_cosine(n)
    t = np.float32(ts[0])
    dt = np.float32(ts[1] - ts[0])
    out = []
    for step in range(1, n + 1):
        out.append((float(t), float(dt)))
        t = np.float32(t + dt)
        if step < n:
            dt = np.float32(ts[step + 1] - t)
    return out


def solve_euler(W, z, mu, spks, cond, mask=None, n_steps=N_TIMESTEPS, capture=None):
    """Batched CFG Euler solve.  z/mu/cond: [U, 80, T]; spks: [U, 80]; mask:
    bool [U, T, T] or None.  Each utterance's conditional row is paired with
    an unconditional row (mu, spks, cond zeroed) at the same x and t
    (flow_reference.py:480-495).  Returns x after the last step [U, 80, T]."""
    dtype = z.dtype
    U = z.shape[0]
    x = z.copy()
    zeros = np.zeros_like(mu)
    mu_in = np.concatenate([mu, zeros], axis=0)
    cond_in = np.concatenate([cond, np.zeros_like(cond)], axis=0)
    spks_in = np.concatenate([spks, np.zeros_like(spks)], axis=0).astype(dtype)
    mask_in = None if mask is None else np.concatenate([mask, mask], axis=0)
    a = dtype.type(1.0 + CFG_RATE)
    b = dtype.type(CFG_RATE)
    for step, (t, dt) in enumerate(euler_schedule(n_steps), start=1):
        x_in = np.concatenate([x, x], axis=0)
        cap = capture if (capture is not None and step == 1) else None
        d = dit_forward(W, x_in, mu_in, np.full((2 * U,), t, np.float32), spks_in, cond_in, mask_in, cap)
        if cap is not None:
            capture["dphi_step1"] = d
        x = (x + dtype.type(dt) * (a * d[:U] - b * d[U:])).astype(dtype)
    return x


# ---------------------------------------------------------------------------
# Frontend (once per utterance): flow_reference.py:406-429, 531-563;
# src/flow/flow.cpp:129-182, prelookahead.cpp:8-20, ops.cpp:106-122
# ---------------------------------------------------------------------------
def conv1d(x, w, b):
    """Plain Conv1d, stride 1, no padding.  x: [C_in, L]; w: [C_out, C_in, K]."""
    K = w.shape[2]
    L = x.shape[1] - K + 1
    cols = np.stack([x[:, k:k + L] for k in range(K)], axis=0)     # [K, C_in, L]
    return np.einsum("ock,kcl->ol", w, cols) + b[:, None]


def prelookahead(W, tok_emb, finalize=True):
    """PreLookaheadLayer (flow_reference.py:406-429).  tok_emb: [Tseq, 80].
    finalize=True: the sequence is right-padded with PRE_LOOKAHEAD zero rows and
    all Tseq rows come out.  finalize=False (the streaming call,
    flow_reference.py:546-548): the last PRE_LOOKAHEAD rows are look-ahead
    context only (they replace the zero padding) and Tseq - PRE_LOOKAHEAD rows
    come out, with the residual taken from the non-context rows."""
    if finalize:
        inp = tok_emb
        x = np.concatenate([tok_emb.T, np.zeros((MEL_DIM, PRE_LOOKAHEAD), tok_emb.dtype)], axis=1)
    else:
        if tok_emb.shape[0] <= PRE_LOOKAHEAD:
            raise ValueError("streaming PreLookahead needs more rows than the look-ahead context")
        inp = tok_emb[:-PRE_LOOKAHEAD]
        x = tok_emb.T                                               # inputs ++ context, no padding left
    y = conv1d(x, W["pre_lookahead_layer.conv1.weight"], W["pre_lookahead_layer.conv1.bias"])
    y = np.where(y >= 0, y, y * y.dtype.type(0.01))
    y = np.concatenate([np.zeros((DIM, 2), y.dtype), y], axis=1)
    y = conv1d(y, W["pre_lookahead_layer.conv2.weight"], W["pre_lookahead_layer.conv2.bias"])
    return y.T + inp


def frontend(W, prompt_tokens, tokens, prompt_feat, spk_embedding, capture=None, finalize=True):
    """Returns (mu [80, MEL_T], cond [80, MEL_T], spks [80]).  MEL_T = 2 Tseq
    (finalize) or 2 (Tseq - PRE_LOOKAHEAD) (streaming; flow_reference.py:531-555)."""
    e = np.asarray(spk_embedding, np.float32).reshape(-1)
    e = e / max(float(np.sqrt((e.astype(np.float64) ** 2).sum())), 1e-12)
    spk = (W["spk_embed_affine_layer.weight"] @ e.astype(np.float32) + W["spk_embed_affine_layer.bias"]).astype(np.float32)
    tok = np.concatenate([np.asarray(prompt_tokens), np.asarray(tokens)]).astype(np.int64)
    tok = np.maximum(tok, 0)
    emb = W["input_embedding.weight"][tok]                          # [Tseq, 80]
    h = prelookahead(W, emb, finalize)
    h = np.repeat(h, TOKEN_MEL_RATIO, axis=0)                       # [MEL_T, 80]
    pf = np.asarray(prompt_feat, np.float32).reshape(-1, MEL_DIM)
    mel_t = h.shape[0]
    cond = np.zeros((mel_t, MEL_DIM), np.float32)
    cond[: pf.shape[0]] = pf
    if capture is not None:
        capture.update(spk=spk, token_embed=emb, prelookahead=h[::TOKEN_MEL_RATIO])
    return np.ascontiguousarray(h.T.astype(np.float32)), np.ascontiguousarray(cond.T), spk


def infer(W, prompt_tokens, tokens, prompt_feat, spk_embedding, noise_z, capture=None, finalize=True):
    """Token -> mel (FlowDecoder::infer 7-arg form, src/flow/flow.cpp:110-287;
    flow_reference.py:531-563 / 598-665).  finalize=False is the streaming
    call (flow_reference.py:546-548).  noise_z: [80, >= MEL_T] (the first MEL_T
    columns are used, as the CFM slices its noise bank,
    flow_reference.py:470).  Returns mel [80, MEL_T - mel_len1]."""
    mu, cond, spk = frontend(W, prompt_tokens, tokens, prompt_feat, spk_embedding, capture, finalize)
    mel_len1 = np.asarray(prompt_feat).reshape(-1, MEL_DIM).shape[0]
    z = np.asarray(noise_z, np.float32).reshape(MEL_DIM, -1)[:, : mu.shape[1]]
    x = solve_euler(W, z[None], mu[None], spk[None], cond[None], None, capture=capture)
    return x[0, :, mel_len1:]


# ---------------------------------------------------------------------------
# Fused-op restatements used by the microbench parity tests
# ---------------------------------------------------------------------------
def op_adaln_mod(x, shift, scale):
    """x: [N, D]; shift/scale: [D] -> LN(x)*(1+scale)+shift."""
    return layer_norm(x) * (x.dtype.type(1.0) + scale) + shift


def op_gate_residual(x, y, gate):
    return x + gate * y


def op_rotary(x, pos):
    """Partial rotary on channels 0..63 of [N, D] rows at positions ``pos``."""
    f = (np.asarray(pos, np.float32)[:, None] * rotary_inv_freq()[None, :]).astype(np.float32)
    f = np.repeat(f, 2, axis=-1)
    cos, sin = np.cos(f).astype(x.dtype), np.sin(f).astype(x.dtype)
    r, u = x[:, :ROT_DIM], x[:, ROT_DIM:]
    return np.concatenate([r * cos + rotate_half(r) * sin, u], axis=-1)
