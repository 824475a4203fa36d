"""flow.gguf tensor inventory and a seeded synthetic-weight writer.

The inventory is the 330 state_dict entries of CosyVoice3's Flow model under
the reference's GGUF names (hardenedlinux/larynx src/flow/gguf.cpp:46-90,
shapes src/flow/internal.h:50-93).  ``write_synthetic_gguf`` streams random
weights (N(0, std), one PCG64 stream per tensor keyed by the CRC-32 of its
name, so any tensor can be regenerated alone) into a GGUF v3 file -- the
benchmark's random-init weights of the real architecture.
"""

from __future__ import annotations

import struct
import zlib
from typing import List, Tuple

import numpy as np

from .gguf import ALIGN, _str

MEL, DIM, FF, DEPTH, VOCAB = 80, 1024, 2048, 22, 6561
EST = "decoder.estimator."


def param_specs() -> List[Tuple[str, Tuple[int, ...]]]:
    s = [
        ("input_embedding.weight", (VOCAB, MEL)),
        ("spk_embed_affine_layer.weight", (MEL, 192)),
        ("spk_embed_affine_layer.bias", (MEL,)),
        ("pre_lookahead_layer.conv1.weight", (DIM, MEL, 4)),
        ("pre_lookahead_layer.conv1.bias", (DIM,)),
        ("pre_lookahead_layer.conv2.weight", (MEL, DIM, 3)),
        ("pre_lookahead_layer.conv2.bias", (MEL,)),
        (EST + "time_embed.time_mlp.0.weight", (DIM, 256)),
        (EST + "time_embed.time_mlp.0.bias", (DIM,)),
        (EST + "time_embed.time_mlp.2.weight", (DIM, DIM)),
        (EST + "time_embed.time_mlp.2.bias", (DIM,)),
        (EST + "input_embed.proj.weight", (DIM, 4 * MEL)),
        (EST + "input_embed.proj.bias", (DIM,)),
        (EST + "input_embed.conv_pos_embed.conv1.0.weight", (DIM, 64, 31)),
        (EST + "input_embed.conv_pos_embed.conv1.0.bias", (DIM,)),
        (EST + "input_embed.conv_pos_embed.conv2.0.weight", (DIM, 64, 31)),
        (EST + "input_embed.conv_pos_embed.conv2.0.bias", (DIM,)),
        (EST + "rotary_embed.inv_freq", (32,)),
    ]
    for i in range(DEPTH):
        b = f"{EST}transformer_blocks.{i}."
        s += [(b + "attn_norm.linear.weight", (6 * DIM, DIM)), (b + "attn_norm.linear.bias", (6 * DIM,))]
        for p in ("to_q", "to_k", "to_v"):
            s += [(b + f"attn.{p}.weight", (DIM, DIM)), (b + f"attn.{p}.bias", (DIM,))]
        s += [(b + "attn.to_out.0.weight", (DIM, DIM)), (b + "attn.to_out.0.bias", (DIM,)),
              (b + "ff.ff.0.0.weight", (FF, DIM)), (b + "ff.ff.0.0.bias", (FF,)),
              (b + "ff.ff.2.weight", (DIM, FF)), (b + "ff.ff.2.bias", (DIM,))]
    s += [(EST + "norm_out.linear.weight", (2 * DIM, DIM)), (EST + "norm_out.linear.bias", (2 * DIM,)),
          (EST + "proj_out.weight", (MEL, DIM)), (EST + "proj_out.bias", (MEL,))]
    return s


def inv_freq() -> np.ndarray:
    ar = np.arange(0, 64, 2).astype(np.float32) / np.float32(64)
    return (np.float32(1.0) / np.power(np.float32(10000.0), ar).astype(np.float32)).astype(np.float32)


def synth_tensor(name: str, shape, seed: int = 0, std: float = 0.02) -> np.ndarray:
    if name.endswith("rotary_embed.inv_freq"):
        return inv_freq()
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    return (rng.standard_normal(tuple(shape), dtype=np.float32) * np.float32(std)).astype(np.float32)


def write_synthetic_gguf(path: str, seed: int = 0, std: float = 0.02) -> None:
    """Stream all 330 tensors (float32) into a GGUF v3 file."""
    specs = param_specs()
    header = bytearray()
    header += b"GGUF" + struct.pack("<I", 3) + struct.pack("<q", len(specs)) + struct.pack("<q", 1)
    header += _str("general.architecture") + struct.pack("<i", 8) + _str("cosyvoice3-flow")
    offset = 0
    for name, shape in specs:
        ne = list(reversed(shape))
        header += _str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}q", *ne)
        header += struct.pack("<i", 0) + struct.pack("<Q", offset)
        nbytes = int(np.prod(shape)) * 4
        offset += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * ((-len(header)) % ALIGN))
        for name, shape in specs:
            a = synth_tensor(name, shape, seed, std)
            f.write(a.tobytes())
            f.write(b"\0" * ((-a.nbytes) % ALIGN))
