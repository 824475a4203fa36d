"""hift.gguf tensor inventory, a seeded synthetic-weight writer and the
SineGen2 source-asset writer.

The inventory is the 246 tensors the reference's HiFT loader resolves by name
(hardenedlinux/larynx src/hift/gguf.cpp:95-128, shapes src/hift/internal.h:
72-120): CosyVoice3's CausalHiFTGenerator with the weight-norm already folded
into plain conv weights, all float32.  Shapes are PyTorch order (the GGUF `ne`
is the reverse).

``write_synthetic_hift_gguf`` writes random weights of that architecture (one
PCG64 stream per tensor keyed by the CRC-32 of its name).  The scales keep the
activations of the random network O(1) through the three upsample stages and
put the f0 predictor's output in the voiced range for part of the frames, so
both branches of SineGen2 are exercised.

``write_source_asset`` writes the "HSRC" v1 file that
``HiftVocoder::load_source`` reads (src/hift/hift.cpp:84-131): u32 magic
0x43525348, u32 version 1, u32 harmonic_dim 9, u64 sine_max (300 s * 24 kHz),
then rand_ini[9] and sine_waves[sine_max][9] as float32.
"""

from __future__ import annotations

import struct
import zlib
from typing import List, Tuple

import numpy as np

from .gguf import ALIGN, _str

IN_CH, BASE_CH, NB_HARM = 80, 512, 8
UPSAMPLE_RATES = (8, 5, 3)
UPSAMPLE_KERNELS = (16, 11, 7)
RESBLOCK_KERNELS = (3, 7, 11)
SRC_RB_KERNELS = (7, 7, 11)
SRC_DOWN_KERNELS = (30, 6, 1)
SAMPLE_RATE = 24000
SINE_MAX_SAMPLES = 300 * SAMPLE_RATE
HSRC_MAGIC = 0x43525348


def stage_channels(i: int) -> int:
    return BASE_CH >> (i + 1)


def _resblock_specs(prefix: str, ch: int, k: int) -> List[Tuple[str, Tuple[int, ...]]]:
    s = []
    for j in range(3):
        s += [(f"{prefix}.convs1.{j}.weight", (ch, ch, k)), (f"{prefix}.convs1.{j}.bias", (ch,)),
              (f"{prefix}.convs2.{j}.weight", (ch, ch, k)), (f"{prefix}.convs2.{j}.bias", (ch,)),
              (f"{prefix}.activations1.{j}.alpha", (ch,)), (f"{prefix}.activations2.{j}.alpha", (ch,))]
    return s


def param_specs() -> List[Tuple[str, Tuple[int, ...]]]:
    s = [("conv_pre.weight", (BASE_CH, IN_CH, 5)), ("conv_pre.bias", (BASE_CH,)),
         ("conv_post.weight", (18, 64, 7)), ("conv_post.bias", (18,))]
    cin = BASE_CH
    for i in range(3):
        ch = stage_channels(i)
        s += [(f"ups.{i}.weight", (ch, cin, UPSAMPLE_KERNELS[i])), (f"ups.{i}.bias", (ch,)),
              (f"source_downs.{i}.weight", (ch, 18, SRC_DOWN_KERNELS[i])), (f"source_downs.{i}.bias", (ch,))]
        s += _resblock_specs(f"source_resblocks.{i}", ch, SRC_RB_KERNELS[i])
        cin = ch
    for i in range(3):
        for j in range(3):
            s += _resblock_specs(f"resblocks.{i * 3 + j}", stage_channels(i), RESBLOCK_KERNELS[j])
    s += [("m_source.l_linear.weight", (1, NB_HARM + 1)), ("m_source.l_linear.bias", (1,))]
    s += [("f0_predictor.condnet.0.weight", (BASE_CH, IN_CH, 4)), ("f0_predictor.condnet.0.bias", (BASE_CH,))]
    for idx in (2, 4, 6, 8):
        s += [(f"f0_predictor.condnet.{idx}.weight", (BASE_CH, BASE_CH, 3)),
              (f"f0_predictor.condnet.{idx}.bias", (BASE_CH,))]
    s += [("f0_predictor.classifier.weight", (1, BASE_CH)), ("f0_predictor.classifier.bias", (1,))]
    return s


def synth_tensor(name: str, shape, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    shape = tuple(shape)
    if name.endswith(".alpha"):
        return rng.uniform(0.5, 1.5, shape).astype(np.float32)
    if name == "f0_predictor.classifier.bias":
        return np.full(shape, 120.0, np.float32)
    if name == "f0_predictor.classifier.weight":
        return (rng.standard_normal(shape) * (400.0 / np.sqrt(shape[1]))).astype(np.float32)
    if name.startswith("m_source"):
        return (rng.standard_normal(shape) * (0.5 if name.endswith("weight") else 0.05)).astype(np.float32)
    if name.endswith(".bias"):
        return (rng.standard_normal(shape) * 0.02).astype(np.float32)
    # conv weight (out, in, k): unit-gain fan-in scaling, smaller for the
    # residual branches and the final projection (exp() of its first half)
    fan_in = int(np.prod(shape[1:]))
    gain = 1.0
    if ".convs" in name:
        gain = 0.5
    elif name.startswith("conv_post"):
        gain = 0.5
    return (rng.standard_normal(shape) * (gain / np.sqrt(fan_in))).astype(np.float32)


def synthetic_weights(seed: int = 0) -> dict:
    return {name: synth_tensor(name, shape, seed) for name, shape in param_specs()}


def write_synthetic_hift_gguf(path: str, seed: int = 0) -> None:
    """All 246 tensors (float32) into a GGUF v3 file."""
    specs = param_specs()
    header = bytearray()
    header += b"GGUF" + struct.pack("<I", 3) + struct.pack("<q", len(specs)) + struct.pack("<q", 1)
    header += _str("general.architecture") + struct.pack("<i", 8) + _str("cosyvoice3.hift")
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
            a = synth_tensor(name, shape, seed)
            f.write(a.tobytes())
            f.write(b"\0" * ((-a.nbytes) % ALIGN))


def synthetic_source(seed: int = 0, n_samples: int = SINE_MAX_SAMPLES):
    """rand_ini [9] (column 0 zero, as SineGen2 builds it) and the first
    n_samples rows of a N(0, 1) unvoiced-noise bank [n_samples][9]."""
    rng = np.random.default_rng([seed, 0x48535243])
    rand_ini = rng.uniform(0.0, 1.0, NB_HARM + 1).astype(np.float32)
    rand_ini[0] = 0.0
    bank = rng.standard_normal((n_samples, NB_HARM + 1), dtype=np.float32)
    return rand_ini, bank


def write_source_asset(path: str, rand_ini: np.ndarray, bank: np.ndarray) -> None:
    rand_ini = np.ascontiguousarray(rand_ini, np.float32).reshape(NB_HARM + 1)
    bank = np.ascontiguousarray(bank, np.float32).reshape(-1, NB_HARM + 1)
    with open(path, "wb") as f:
        f.write(struct.pack("<III", HSRC_MAGIC, 1, NB_HARM + 1) + struct.pack("<Q", bank.shape[0]))
        f.write(rand_ini.tobytes())
        f.write(bank.tobytes())
