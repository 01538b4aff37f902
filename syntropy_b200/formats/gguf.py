"""GGUF reading (native header parser): metadata, tensor infos, and tensor data in F32 / F16 /
BF16 and the Q8_0 / Q4_0 / Q4_1 / Q4_K / Q6_K block formats (dequantised to f32).  Q4_1 blocks
map 1:1 onto this framework's 4-bit interchange layout.
Reference: crates/manifest/src/gguf.rs:75-335."""
from __future__ import annotations

import mmap

import numpy as np
import torch

from .._ext import ext

from .ggml_blocks import BLOCKS, DEQUANT, GGML_TYPE

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0, GGML_BF16 = 0, 1, 2, 3, 8, 30
_BLOCK = {t: BLOCKS[n] for t, n in GGML_TYPE.items()}


class GGUFFile:
    def __init__(self, path: str):
        self.path = path
        self.version, meta, tensors, self.data_start = ext().gguf_header(path)
        self.meta = dict(meta)
        self.tensors = {n: (t, tuple(int(d) for d in dims), int(off)) for n, t, dims, off in tensors}
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)

    def nbytes(self, name: str) -> int:
        t, dims, _ = self.tensors[name]
        n = int(np.prod(dims))
        bs, bb = _BLOCK[t]
        return n // bs * bb

    def raw(self, name: str) -> torch.Tensor:
        t, dims, off = self.tensors[name]
        b = self.data_start + off
        return torch.frombuffer(memoryview(self._mm)[b: b + self.nbytes(name)], dtype=torch.uint8).clone()

    def get(self, name: str) -> torch.Tensor:
        """Dense f32 tensor with torch shape (GGUF dims are innermost-first)."""
        t, dims, _ = self.tensors[name]
        return self._decode(name, t, self.raw(name), tuple(reversed(dims)))

    def get_row(self, name: str, i: int) -> torch.Tensor:
        """Row `i` of the outermost dimension (one expert of a stacked tensor), read and
        dequantised alone; a row is a whole number of blocks, so it starts on a block."""
        t, dims, off = self.tensors[name]
        shape = tuple(reversed(dims))
        if not 0 <= i < shape[0]:
            raise IndexError(f"{name}: row {i} of {shape[0]}")
        per = self.nbytes(name) // shape[0]
        b = self.data_start + off + i * per
        r = torch.frombuffer(memoryview(self._mm)[b: b + per], dtype=torch.uint8).clone()
        return self._decode(name, t, r, shape[1:])

    @staticmethod
    def _decode(name: str, t: int, r: torch.Tensor, shape: tuple) -> torch.Tensor:
        if t == GGML_F32:
            return r.view(torch.float32).reshape(shape)
        if t == GGML_F16:
            return r.view(torch.float16).float().reshape(shape)
        if t == GGML_BF16:
            return r.view(torch.bfloat16).float().reshape(shape)
        if GGML_TYPE.get(t) in DEQUANT:  # native, multi-threaded over blocks
            return ext().ggml_dequant(r.contiguous(), GGML_TYPE[t]).reshape(shape)
        raise NotImplementedError(f"GGML type {t} for {name}")

    def close(self):
        self._mm.close()
        self._f.close()


def write_gguf(path: str, tensors: dict, meta: dict | None = None, alignment: int = 32):
    """Minimal GGUF v3 writer (F32 tensors and Q4_1 row blocks) for fixtures."""
    import struct

    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    meta = dict(meta or {})
    meta["general.alignment"] = alignment
    out = bytearray(b"GGUF" + struct.pack("<I", 3) + struct.pack("<QQ", len(tensors), len(meta)))
    for k, v in meta.items():
        out += s(k)
        if isinstance(v, bool):
            out += struct.pack("<IB", 7, int(v))
        elif isinstance(v, int):
            out += struct.pack("<IQ", 10, v) if v >= 0 else struct.pack("<Iq", 11, v)
        elif isinstance(v, float):
            out += struct.pack("<Id", 12, v)
        else:
            out += struct.pack("<I", 8) + s(str(v))
    blobs, off = [], 0
    for n, (kind, t) in tensors.items():
        if kind == "q4_1":
            rows, shape = t
            raw, gtype = rows.numpy().tobytes(), GGML_Q4_1
        else:
            shape, raw, gtype = tuple(t.shape), t.float().contiguous().numpy().tobytes(), GGML_F32
        out += s(n) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in reversed(shape))
        out += struct.pack("<IQ", gtype, off)
        pad = (-len(raw)) % alignment
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    out += b"\0" * ((-len(out)) % alignment)
    with open(path, "wb") as f:
        f.write(out)
        for b in blobs:
            f.write(b)
