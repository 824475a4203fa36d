"""GGUF v3 writer/reader (little-endian), enough for flow.gguf.

Layout (hardenedlinux/larynx docs/WEIGHT_FORMAT.md:15-110): "GGUF", u32
version 3, i64 n_tensors, i64 n_kv, KV section, tensor infos (name, u32
n_dims, i64 ne[] = reversed torch shape, i32 ggml type, u64 offset into the
data blob), padding to 32 bytes, data blob with every tensor padded to 32.
Used by the tests and the benchmark to write seeded synthetic weights under
the reference's tensor names; the C++ loader (csrc/gguf.cpp) reads it.
"""

from __future__ import annotations

import struct
from typing import Dict, Iterable, Tuple

import numpy as np

ALIGN = 32
GGML_TYPES = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str, tensors: Iterable[Tuple[str, np.ndarray]], kv: Dict[str, str] | None = None) -> None:
    tensors = [(n, np.ascontiguousarray(a)) for n, a in tensors]
    kv = kv or {}
    header = bytearray()
    header += b"GGUF" + struct.pack("<I", 3) + struct.pack("<q", len(tensors)) + struct.pack("<q", len(kv))
    for k, v in kv.items():
        header += _str(k) + struct.pack("<i", 8) + _str(v)
    offset = 0
    offsets = []
    for name, a in tensors:
        if a.dtype not in GGML_TYPES:
            raise ValueError(f"unsupported dtype {a.dtype} for {name}")
        ne = list(reversed(a.shape)) or [1]
        header += _str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}q", *ne)
        header += struct.pack("<i", GGML_TYPES[a.dtype]) + struct.pack("<Q", offset)
        offsets.append(offset)
        offset += (a.nbytes + ALIGN - 1) // ALIGN * ALIGN
    pad = (-len(header)) % ALIGN
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * pad)
        for (name, a), off in zip(tensors, offsets):
            f.write(a.tobytes())
            f.write(b"\0" * ((-a.nbytes) % ALIGN))


def read_gguf_index(path: str):
    """Returns {name: (torch_shape, ggml_type)} (for tests)."""
    with open(path, "rb") as f:
        data = f.read(1 << 22)
    p = 0

    def get(fmt):
        nonlocal p
        v = struct.unpack_from(fmt, data, p)
        p += struct.calcsize(fmt)
        return v[0]

    def gstr():
        nonlocal p
        n = get("<Q")
        s = data[p:p + n].decode()
        p += n
        return s

    assert data[:4] == b"GGUF"
    p = 4
    get("<I")
    nt = get("<q")
    nkv = get("<q")
    for _ in range(nkv):
        gstr()
        t = get("<i")
        assert t == 8, "only string KVs are written by this module"
        gstr()
    out = {}
    for _ in range(nt):
        name = gstr()
        nd = get("<I")
        ne = [get("<q") for _ in range(nd)]
        ty = get("<i")
        get("<Q")
        out[name] = (tuple(reversed(ne)), ty)
    return out


def write_noise_bank(path: str, bank: np.ndarray) -> None:
    """FNSE asset (tests/export_flow_noise.py:15-20 of the reference):
    u32 magic 0x45534E46, u32 version 1, u32 mel_dim, u64 max_frames,
    f32[mel_dim][max_frames]."""
    bank = np.ascontiguousarray(bank, dtype=np.float32)
    with open(path, "wb") as f:
        f.write(struct.pack("<IIIQ", 0x45534E46, 1, bank.shape[0], bank.shape[1]))
        f.write(bank.tobytes())
