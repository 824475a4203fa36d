"""The reference's own stage-dump driver on the B200 library.

oracle/_ref/larynx_flow_dump is the reference's tests/flow_dump.cpp,
unchanged, compiled against the reference's include/larynx/flow/flow.h and
linked with larynx_b200/shim/flow_decoder.cpp (FlowDecoder over the C ABI)
by oracle/Makefile.  Fed the inputs of the reference's 24-frame validation
case (the files tests/verify_flow.py writes from flow_ref.npz), it must write
every stage file verify_flow.py reads, with the sizes it asserts, and each
stage must pass verify_flow.py's gate (max|d| / max|ref| <= 1e-2) against the
golden vectors the reference produced (the 22 blocks: the golden where it
holds them, the oracle's step-1 captures for all).  Skipped where the driver
was not built (no reference checkout on the build machine)."""

import os
import subprocess

import numpy as np
import pytest

from conftest import REPO, golden, rel_max

DUMP = os.path.join(REPO, "oracle", "_ref", "larynx_flow_dump")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(DUMP), reason="oracle/_ref/larynx_flow_dump not built")]
GATE = 1e-2

# tests/verify_flow.py:37-50 -- (stage file, golden key, shape)
STAGES = (("spk.f32", "spk", (1, 80)), ("token_embed.f32", "token_embed", (1, 12, 80)),
          ("prelookahead.f32", "prelookahead", (1, 12, 80)), ("mu.f32", "mu", (1, 80, 24)),
          ("cond.f32", "cond", (1, 80, 24)), ("time_embed.f32", "time_embed_step1", (2, 1024)),
          ("input_proj.f32", "dit_input_proj_step1", (2, 24, 1024)),
          ("conv_pos.f32", "dit_conv_pos_step1", (2, 24, 1024)),
          ("input_embed.f32", "dit_input_embed_step1", (2, 24, 1024)),
          ("norm_out.f32", "dit_norm_out_step1", (2, 24, 1024)), ("dphi.f32", "dphi_step1", (2, 80, 24)),
          ("feat.f32", "feat", (1, 80, 16)))


def _load(path, shape):
    a = np.fromfile(path, dtype=np.float32)
    assert a.size == int(np.prod(shape)), (path, a.size, shape)
    return a.reshape(shape)


def test_reference_dump_driver_stages(tmp_path, weights):
    from larynx_b200.weights import write_synthetic_gguf
    from oracle import flow_oracle as fo
    g = golden("flow_fixture.npz")
    gguf = str(tmp_path / "flow.gguf")
    write_synthetic_gguf(gguf, seed=0, std=0.02)
    indir, outdir = tmp_path / "in", tmp_path / "out"
    indir.mkdir()
    outdir.mkdir()
    g["prompt_tokens"].astype(np.int32).reshape(-1).tofile(indir / "prompt_tokens.i32")
    g["tokens"].astype(np.int32).reshape(-1).tofile(indir / "tokens.i32")
    for k in ("prompt_feat", "spk_embedding", "noise_z"):
        g[k].astype(np.float32).reshape(-1).tofile(indir / f"{k}.f32")
    r = subprocess.run([DUMP, gguf, str(indir), str(outdir)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    for fname, key, shape in STAGES:
        assert rel_max(_load(outdir / fname, shape), g[key]) <= GATE, fname
    cap = {}
    fo.infer(weights, g["prompt_tokens"][0], g["tokens"][0], g["prompt_feat"][0], g["spk_embedding"][0],
             g["noise_z"][0], capture=cap)
    for i in range(22):
        blk = _load(outdir / f"block{i}.f32", (2, 24, 1024))
        assert rel_max(blk, cap["blocks"][i]) <= GATE, i
        if f"dit_block{i}" in g.files:
            assert rel_max(blk, g[f"dit_block{i}"]) <= GATE, i
