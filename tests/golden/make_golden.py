#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ from the reference itself.

Imports hardenedlinux/larynx's own ground-truth Flow model,
``tests/flow_reference.py`` (from the reference checkout named by
$LARYNX_REF, which is required), loads the seeded synthetic weights of
``oracle.flow_oracle.synth_weights`` (seed 0, N(0, 0.02); the rotary
``inv_freq`` buffer keeps its formula value) and records:

  flow_fixture.npz  the reference's own validation case (4 prompt tokens + 8
                    tokens -> 24 mel frames -> 16 output frames, input seed
                    1234, CFM noise = seed-0 bank; flow_reference.py:42-47,
                    668-704), per-stage captures at CFM step 1 and the final mel
  dit_padded.npz    one estimator forward on a padded batch (lengths 20, 32,
                    key-padding mask, non-streaming path) plus a 10-step CFG
                    solve of the same batch driven by a loop that mirrors
                    solve_euler (flow_reference.py:476-501)
  dit_chunk.npz     one estimator forward with a block-causal chunk mask
                    (chunk 50) through the streaming [B, T, T] mask input
                    (flow_reference.py:375-376)
  flow_stream.npz   the streaming call (finalize=False: PreLookahead with the
                    last 3 tokens as context) and the finalize=True output
                    of the same inputs
  ops_fixture.npz   the fused-op pieces (AdaLN-Zero modulation, partial
                    rotary, GELU-tanh, Mish, time embedding + modulation
                    chunks for the 10-step schedule)

Run once in a container where the reference is readable:
    LARYNX_REF=<reference checkout> python tests/golden/make_golden.py
The GPU box never runs this script; it only reads the .npz files.
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import flow_oracle as fo  # noqa: E402

REF = os.environ.get("LARYNX_REF")
if not REF:
    sys.exit("set LARYNX_REF to the reference checkout (the folder holding tests/flow_reference.py)")
sys.path.insert(0, os.path.join(REF, "tests"))
import flow_reference as fr  # noqa: E402

KEEP_BLOCKS = (0, 10, 21)


def load_model():
    torch.set_num_threads(os.cpu_count() or 1)
    model = fr.build_model().eval()
    W = fo.synth_weights(seed=0, std=0.02)
    sd = {k: torch.from_numpy(v.copy()) for k, v in W.items()}
    model.load_state_dict(sd, strict=True)
    return model, W


def make_flow_fixture(model):
    torch.manual_seed(fr.INPUT_SEED)
    prompt_tokens = torch.randint(0, fr.VOCAB, (1, fr.P))
    tokens = torch.randint(0, fr.VOCAB, (1, fr.T))
    prompt_feat = torch.randn(1, fr.MEL_LEN1, 80)
    spk_embedding = torch.randn(1, 192)
    cap = {}
    with torch.inference_mode():
        feat = fr.manual_inference(model, prompt_tokens, tokens, prompt_feat, spk_embedding, cap)
        feat_model, _ = model.inference(tokens, torch.tensor([fr.T]), prompt_tokens, torch.tensor([fr.P]),
                                        prompt_feat, torch.tensor([fr.MEL_LEN1]), spk_embedding,
                                        streaming=False, finalize=True)
    assert (feat - feat_model).abs().max().item() < 1e-5
    out = {
        "prompt_tokens": prompt_tokens.numpy().astype(np.int32),
        "tokens": tokens.numpy().astype(np.int32),
        "prompt_feat": prompt_feat.numpy(),
        "spk_embedding": spk_embedding.numpy(),
        "noise_z": cap["noise_z"].numpy(),
        "spk": cap["spk"].numpy(),
        "token_embed": cap["token_embed"].numpy(),
        "prelookahead": cap["prelookahead"].numpy(),
        "mu": cap["mu"].numpy(),
        "cond": cap["cond"].numpy(),
        "t_span": cap["t_span"].numpy(),
        "time_embed_step1": cap["time_embed"].numpy(),
        "dit_input_proj_step1": cap["input_proj"].numpy(),
        "dit_conv_pos_step1": cap["conv_pos"].numpy(),
        "dit_input_embed_step1": cap["input_embed"].numpy(),
        "dit_norm_out_step1": cap["norm_out"].numpy(),
        "dphi_step1": cap["dphi_step1"].numpy(),
        "feat": feat.numpy(),
    }
    for i in KEEP_BLOCKS:
        out[f"dit_block{i}"] = cap["blocks"][i].numpy()
    np.savez_compressed(os.path.join(HERE, "flow_fixture.npz"), **out)


def make_stream(model):
    """The streaming (finalize=False) call of the reference's flow inference
    (flow_reference.py:531-563): 4 prompt tokens + 12 tokens, the last 3
    tokens acting as PreLookahead context; also the finalize=True output of
    the same inputs."""
    torch.manual_seed(4321)
    P, T = 4, 12
    prompt_tokens = torch.randint(0, fr.VOCAB, (1, P))
    tokens = torch.randint(0, fr.VOCAB, (1, T))
    prompt_feat = torch.randn(1, 2 * P, 80)
    spk_embedding = torch.randn(1, 192)
    args = (tokens, torch.tensor([T]), prompt_tokens, torch.tensor([P]), prompt_feat, torch.tensor([2 * P]),
            spk_embedding)
    with torch.inference_mode():
        feat_s, _ = model.inference(*args, streaming=False, finalize=False)
        feat_s2, _ = model.inference(*args, streaming=True, finalize=False)
        feat_f, _ = model.inference(*args, streaming=False, finalize=True)
        tok = torch.concat([prompt_tokens, tokens], dim=1)
        emb = model.input_embedding(torch.clamp(tok, min=0))
        pre = model.pre_lookahead_layer(emb[:, :-model.pre_lookahead_len], context=emb[:, -model.pre_lookahead_len:])
    assert (feat_s - feat_s2).abs().max().item() < 1e-6  # streaming mask == padding mask at batch 1
    mel_t = 2 * (P + T - 3)
    np.savez_compressed(os.path.join(HERE, "flow_stream.npz"),
                        prompt_tokens=prompt_tokens.numpy().astype(np.int32), tokens=tokens.numpy().astype(np.int32),
                        prompt_feat=prompt_feat.numpy(), spk_embedding=spk_embedding.numpy(),
                        noise_z=model.decoder.rand_noise[:, :, :2 * (P + T)].numpy(),
                        prelookahead=pre.numpy(), feat_stream=feat_s.numpy(), feat_final=feat_f.numpy(),
                        mel_t=np.int32(mel_t))


def make_padded(model):
    g = torch.Generator().manual_seed(7)
    lengths = [20, 32]
    B, T = len(lengths), max(lengths)
    x = torch.randn(B, 80, T, generator=g)
    mu = torch.randn(B, 80, T, generator=g)
    spks = torch.randn(B, 80, generator=g)
    cond = torch.randn(B, 80, T, generator=g)
    for b, L in enumerate(lengths):
        cond[b, :, int(0.2 * L):] = 0
        x[b, :, L:] = 0
        mu[b, :, L:] = 0
        cond[b, :, L:] = 0
    mask = (~fr.make_pad_mask(torch.tensor(lengths), T)).float().unsqueeze(1)  # [B,1,T]
    t = torch.full((B,), 0.3)
    est = model.decoder.estimator
    with torch.inference_mode():
        dphi = est(x, mask, mu, t, spks, cond, streaming=False)
        # 10-step CFG solve of the padded batch, mirroring solve_euler
        t_span = 1 - torch.cos(torch.linspace(0, 1, 11) * 0.5 * torch.pi)
        z = x.clone()
        tt, dt = t_span[0], t_span[1] - t_span[0]
        xs = z
        for step in range(1, 11):
            x_in = torch.cat([xs, xs], 0)
            mask_in = torch.cat([mask, mask], 0)
            mu_in = torch.cat([mu, torch.zeros_like(mu)], 0)
            spk_in = torch.cat([spks, torch.zeros_like(spks)], 0)
            cond_in = torch.cat([cond, torch.zeros_like(cond)], 0)
            d = est(x_in, mask_in, mu_in, tt.repeat(2 * B), spk_in, cond_in, streaming=False)
            dc, du = torch.split(d, [B, B], 0)
            xs = xs + dt * ((1.0 + 0.7) * dc - 0.7 * du)
            tt = tt + dt
            if step < 10:
                dt = t_span[step + 1] - tt
    np.savez_compressed(os.path.join(HERE, "dit_padded.npz"), lengths=np.array(lengths, np.int32),
                        x=x.numpy(), mu=mu.numpy(), spks=spks.numpy(), cond=cond.numpy(), t=np.float32(0.3),
                        dphi=dphi.numpy(), solve=xs.numpy())


def make_chunk(model):
    g = torch.Generator().manual_seed(11)
    lengths = [120, 96]
    chunk = 50
    B, T = len(lengths), max(lengths)
    x = torch.randn(B, 80, T, generator=g)
    mu = torch.randn(B, 80, T, generator=g)
    spks = torch.randn(B, 80, generator=g)
    cond = torch.zeros(B, 80, T)
    for b, L in enumerate(lengths):
        x[b, :, L:] = 0
        mu[b, :, L:] = 0
    m = torch.from_numpy(fo.block_causal_mask(lengths, T, chunk)).float()  # [B, T, T]
    t = torch.full((B,), 0.55)
    with torch.inference_mode():
        dphi = model.decoder.estimator(x, m, mu, t, spks, cond, streaming=True)
    np.savez_compressed(os.path.join(HERE, "dit_chunk.npz"), lengths=np.array(lengths, np.int32), chunk=np.int32(chunk),
                        x=x.numpy(), mu=mu.numpy(), spks=spks.numpy(), cond=cond.numpy(), t=np.float32(0.55),
                        dphi=dphi.numpy())


def make_ops(model):
    g = torch.Generator().manual_seed(1)
    N, D = 64, 1024
    x = torch.randn(N, D, generator=g)
    mod = torch.randn(2, 6 * D, generator=g) * 0.5
    shift, scale = mod[0, :D], mod[0, D:2 * D]
    ln = torch.nn.LayerNorm(D, elementwise_affine=False, eps=1e-6)
    adaln = ln(x) * (1 + scale) + shift
    rot = fr.RotaryEmbedding(64)
    pos = torch.arange(N) * 23 + 5                    # scattered positions up to ~1500
    freqs, _ = rot.forward(pos)
    rotary = fr.apply_rotary_pos_emb(x.unsqueeze(0), freqs, 1.0)[0]
    gelu = torch.nn.GELU(approximate="tanh")(x * 3)
    mish = torch.nn.Mish()(x * 3)
    est = model.decoder.estimator
    t_span = 1 - torch.cos(torch.linspace(0, 1, 11) * 0.5 * torch.pi)
    with torch.inference_mode():
        temb = est.time_embed(t_span[:10].clone())
        mod0 = est.transformer_blocks[0].attn_norm.linear(torch.nn.functional.silu(temb))
        modf = est.norm_out.linear(torch.nn.functional.silu(temb))
    np.savez_compressed(os.path.join(HERE, "ops_fixture.npz"), x=x.numpy(), mod=mod.numpy(), adaln=adaln.numpy(),
                        pos=pos.numpy().astype(np.int32), rotary=rotary.numpy(), gelu=gelu.numpy(), mish=mish.numpy(),
                        t_span=t_span.numpy(), temb=temb.numpy(), mod_block0=mod0.numpy(), mod_final=modf.numpy())


def main():
    model, _ = load_model()
    make_ops(model)
    make_chunk(model)
    make_padded(model)
    make_flow_fixture(model)
    make_stream(model)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
