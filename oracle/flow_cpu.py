"""Multithreaded CPU restatement of the Flow decode, for the timed CPU baseline
(TEST INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and its
``--impl reference`` arm time it; tests/ check it against the numpy oracle;
the product path never imports it).

The numpy oracle (``flow_oracle.py``) is the parity checker: it follows the
reference's PyTorch model (``tests/flow_reference.py``) operation by operation,
but numpy runs its element-wise work (exp, tanh, softmax) on one thread, so it
is several times slower than the reference's own PyTorch model on the same
cores.  A baseline that slow would overstate the GPU's advantage.  This module
states the same computation with torch CPU operators, which use every host
thread as the reference's model does:

  * time embedding, AdaLN-Zero chunk orders, LayerNorm eps 1e-6 without
    affine (flow_reference.py:125-194, 294-304);
  * input embedding concat order [x, cond, mu, spks], causal grouped conv
    position embedding (k=31, 16 groups, left pad 30, Mish) added to the
    projection (flow_reference.py:140-166, 310-330);
  * partial GPT-J rotary on channels 0..63 before the head split
    (flow_reference.py:52-106, 217-221), softmax attention with a boolean
    mask, padded query rows zeroed after to_out (flow_reference.py:210-249);
  * GELU-tanh feed-forward (flow_reference.py:197-207), final AdaLN with
    scale before shift and proj_out (flow_reference.py:183-194, 394-397);
  * the cosine-schedule CFG Euler solver with t accumulated in float32
    (flow_reference.py:468-501).
All arithmetic is float32.
"""

from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np
import torch
import torch.nn.functional as F

from oracle import flow_oracle as fo

EST = fo.EST


class FlowCPU:
    """The DiT estimator and CFG Euler solve on the host, float32."""

    def __init__(self, W: Dict[str, np.ndarray]):
        self.W = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)) for k, v in W.items()}
        self.inv_freq = torch.from_numpy(fo.rotary_inv_freq())

    def time_embed(self, t: torch.Tensor) -> torch.Tensor:
        half = 128
        e = math.log(10000) / (half - 1)
        freqs = torch.exp(torch.arange(half, dtype=torch.float32) * -e)
        ang = 1000.0 * t[:, None] * freqs[None, :]
        h = torch.cat([torch.sin(ang), torch.cos(ang)], dim=-1)
        W = self.W
        h = F.linear(h, W[EST + "time_embed.time_mlp.0.weight"], W[EST + "time_embed.time_mlp.0.bias"])
        return F.linear(F.silu(h), W[EST + "time_embed.time_mlp.2.weight"], W[EST + "time_embed.time_mlp.2.bias"])

    def conv_pos(self, x: torch.Tensor) -> torch.Tensor:
        """x [B, T, D] -> 2 x (left pad 30, grouped conv k=31, Mish)."""
        p = EST + "input_embed.conv_pos_embed."
        h = x.transpose(1, 2)
        for c in ("conv1.0", "conv2.0"):
            h = F.mish(F.conv1d(F.pad(h, (fo.CONV_POS_KERNEL - 1, 0)), self.W[p + c + ".weight"],
                                self.W[p + c + ".bias"], groups=fo.CONV_POS_GROUPS))
        return h.transpose(1, 2)

    def rotary(self, x: torch.Tensor, T: int) -> torch.Tensor:
        f = torch.arange(T, dtype=torch.float32)[:, None] * self.inv_freq[None, :]
        f = f.repeat_interleave(2, dim=-1)
        cos, sin = torch.cos(f), torch.sin(f)
        r, u = x[..., :fo.ROT_DIM], x[..., fo.ROT_DIM:]
        r2 = r.reshape(*r.shape[:-1], fo.ROT_DIM // 2, 2)
        rh = torch.stack((-r2[..., 1], r2[..., 0]), dim=-1).reshape(r.shape)
        return torch.cat([r * cos + rh * sin, u], dim=-1)

    def dit_forward(self, x, mu, t, spks, cond, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x/mu/cond [B, 80, T], t [B], spks [B, 80], mask bool [B, T, T]
        (True = attend) or None.  Returns dphi [B, 80, T]."""
        W = self.W
        B, _, T = x.shape
        temb = self.time_embed(t)
        st = F.silu(temb)
        cat = torch.cat([x.transpose(1, 2), cond.transpose(1, 2), mu.transpose(1, 2),
                         spks[:, None, :].expand(B, T, fo.MEL_DIM)], dim=-1)
        xe = F.linear(cat, W[EST + "input_embed.proj.weight"], W[EST + "input_embed.proj.bias"])
        h = self.conv_pos(xe) + xe
        amask = None if mask is None else mask[:, None, :, :]
        row_keep = None if mask is None else mask[:, -1, :][:, :, None]
        for i in range(fo.DEPTH):
            b = f"{EST}transformer_blocks.{i}."
            emb = F.linear(st, W[b + "attn_norm.linear.weight"], W[b + "attn_norm.linear.bias"])
            sh_msa, sc_msa, g_msa, sh_mlp, sc_mlp, g_mlp = emb.chunk(6, dim=-1)
            n = F.layer_norm(h, (fo.DIM,), eps=fo.LN_EPS) * (1 + sc_msa[:, None]) + sh_msa[:, None]
            q = self.rotary(F.linear(n, W[b + "attn.to_q.weight"], W[b + "attn.to_q.bias"]), T)
            k = self.rotary(F.linear(n, W[b + "attn.to_k.weight"], W[b + "attn.to_k.bias"]), T)
            v = F.linear(n, W[b + "attn.to_v.weight"], W[b + "attn.to_v.bias"])
            sp = lambda z: z.view(B, T, fo.HEADS, fo.HEAD_DIM).transpose(1, 2)
            o = F.scaled_dot_product_attention(sp(q), sp(k), sp(v), attn_mask=amask)
            o = o.transpose(1, 2).reshape(B, T, fo.DIM)
            o = F.linear(o, W[b + "attn.to_out.0.weight"], W[b + "attn.to_out.0.bias"])
            if row_keep is not None:
                o = o * row_keep
            h = h + g_msa[:, None] * o
            n = F.layer_norm(h, (fo.DIM,), eps=fo.LN_EPS) * (1 + sc_mlp[:, None]) + sh_mlp[:, None]
            f = F.gelu(F.linear(n, W[b + "ff.ff.0.0.weight"], W[b + "ff.ff.0.0.bias"]), approximate="tanh")
            h = h + g_mlp[:, None] * F.linear(f, W[b + "ff.ff.2.weight"], W[b + "ff.ff.2.bias"])
        emb = F.linear(st, W[EST + "norm_out.linear.weight"], W[EST + "norm_out.linear.bias"])
        scale, shift = emb.chunk(2, dim=-1)
        h = F.layer_norm(h, (fo.DIM,), eps=fo.LN_EPS) * (1 + scale[:, None]) + shift[:, None]
        return F.linear(h, W[EST + "proj_out.weight"], W[EST + "proj_out.bias"]).transpose(1, 2)

    def solve_euler(self, z, mu, spks, cond, mask=None, n_steps: int = fo.N_TIMESTEPS) -> torch.Tensor:
        """CFG Euler solve of U utterances: z/mu/cond [U, 80, T], spks [U, 80]."""
        U = z.shape[0]
        x = z.clone()
        mu_in = torch.cat([mu, torch.zeros_like(mu)])
        cond_in = torch.cat([cond, torch.zeros_like(cond)])
        spks_in = torch.cat([spks, torch.zeros_like(spks)])
        mask_in = None if mask is None else torch.cat([mask, mask])
        for t, dt in fo.euler_schedule(n_steps):
            d = self.dit_forward(torch.cat([x, x]), mu_in, torch.full((2 * U,), t), spks_in, cond_in, mask_in)
            x = x + dt * ((1.0 + fo.CFG_RATE) * d[:U] - fo.CFG_RATE * d[U:])
        return x
