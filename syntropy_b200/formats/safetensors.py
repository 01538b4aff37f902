"""safetensors reading (native header parser, memory-mapped tensor data) and writing.

Weights in the 4-bit format are stored as uint8 tensors named ``<name>.q4`` holding the
GGUF Q4_1 row blocks, with the logical shape in the header metadata
(``q4:<name>`` -> "N,K").  Reference: crates/manifest/src/safetensors.rs:143-235."""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np
import torch

from .._ext import ext

_DT = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "U8": torch.uint8, "I8": torch.int8,
       "I32": torch.int32, "I64": torch.int64, "F8_E4M3": torch.float8_e4m3fn, "BOOL": torch.bool}
_DT_NAME = {v: k for k, v in _DT.items()}


class SafetensorsFile:
    def __init__(self, path: str):
        self.path = path
        hlen, tensors, meta = ext().safetensors_header(path)
        self.data_start = 8 + hlen
        self.meta = dict(meta)
        self.tensors = {n: (dt, tuple(sh), b, e) for n, dt, sh, b, e in tensors}
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)

    def keys(self):
        return self.tensors.keys()

    def get(self, name: str) -> torch.Tensor:
        dt, shape, b, e = self.tensors[name]
        dtype = _DT[dt]
        buf = memoryview(self._mm)[self.data_start + b: self.data_start + e]
        t = torch.frombuffer(bytearray(buf), dtype=torch.uint8)
        return t.view(dtype).reshape(shape) if dtype != torch.uint8 else t.reshape(shape)

    def get_row(self, name: str, i: int) -> torch.Tensor:
        """Row `i` of the first dimension, read alone (one expert of a stacked tensor)."""
        dt, shape, b, e = self.tensors[name]
        dtype = _DT[dt]
        n = (e - b) // shape[0]
        if not 0 <= i < shape[0]:
            raise IndexError(f"{name}: row {i} of {shape[0]}")
        buf = memoryview(self._mm)[self.data_start + b + i * n: self.data_start + b + (i + 1) * n]
        t = torch.frombuffer(bytearray(buf), dtype=torch.uint8)
        return t.view(dtype).reshape(shape[1:]) if dtype != torch.uint8 else t.reshape(shape[1:])

    def close(self):
        self._mm.close()
        self._f.close()


def save_file(tensors: dict, path: str, metadata: dict | None = None):
    hdr, off, blobs = {}, 0, []
    for n, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.uint8 else t.numpy().tobytes()
        hdr[n] = {"dtype": _DT_NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    if metadata:
        hdr["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def load_state_dict(path: str) -> dict:
    """All tensors of a file or of every *.safetensors in a directory (q4 tensors are
    dequantised to f32 for the canonical state dict)."""
    from .q4 import dequant_rows_ref
    files = [path] if os.path.isfile(path) else sorted(
        os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
    sd = {}
    for p in files:
        st = SafetensorsFile(p)
        for n in st.keys():
            t = st.get(n)
            if n.endswith(".q4"):
                N, K = (int(x) for x in st.meta[f"q4:{n[:-3]}"].split(","))
                sd[n[:-3]] = dequant_rows_ref(t, N, K)
            else:
                sd[n] = t
        st.close()
    return sd
