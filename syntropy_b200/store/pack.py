"""Packs: prepared (device-format) tensors stored as 4 KiB-aligned extents of one file, with a
JSON sidecar naming each extent (offset, bytes, dtype, shape, BLAKE3 digest).  A restart reads
a pack straight back instead of converting the weights again; the reads go through the native
I/O pool (pread worker threads, O_DIRECT when offset, length and buffer are 4 KiB-aligned)
into aligned bounce buffers, then into the destination tensors (pinned host tiers included).

Reference: plan/rfcs/RFC-0041-model-formats-packs-weight-distribution.md §5 (packs: aligned
extents plus a sidecar, verified by digest) and crates/io/src/pool/linux.rs (the pread pool,
direct I/O alignment contract).
"""
from __future__ import annotations

import json
import os

import torch

from .._ext import ext

ALIGN = 4096
VERSION = 1
CHUNK = 64 << 20  # bytes per I/O job


def _pad(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _bytes_view(t: torch.Tensor) -> torch.Tensor:
    return t.detach().contiguous().view(-1).view(torch.uint8)


def write_pack(path: str, tensors: dict[str, torch.Tensor]) -> dict:
    """Writes every tensor (host or device) as an aligned extent; returns the sidecar."""
    side = {"version": VERSION, "align": ALIGN, "extents": {}}
    off = 0
    with open(path, "wb") as f:
        for name, t in tensors.items():
            b = _bytes_view(t.to("cpu"))
            n = b.numel()
            data = b.numpy().tobytes()
            f.write(data)
            f.write(b"\0" * (_pad(n) - n))
            side["extents"][name] = {"offset": off, "nbytes": n, "dtype": str(t.dtype).replace("torch.", ""),
                                     "shape": list(t.shape), "blake3": ext().blake3(data).hex()}
            off += _pad(n)
    with open(path + ".json", "w") as f:
        json.dump(side, f, indent=1)
    return side


def read_sidecar(path: str) -> dict:
    with open(path + ".json") as f:
        side = json.load(f)
    if side.get("version") != VERSION or side.get("align") != ALIGN:
        raise ValueError(f"{path}: unsupported pack sidecar")
    return side


def read_pack_into(path: str, targets: dict[str, torch.Tensor], threads: int = 8, verify: bool = True) -> int:
    """Fills each target tensor from its extent (shape and dtype must match the sidecar).
    Returns the bytes read.  verify: check every extent's BLAKE3 digest."""
    side = read_sidecar(path)
    pool = ext().IoPool(threads)
    total = 0
    for name, dst in targets.items():
        e = side["extents"].get(name)
        if e is None:
            raise KeyError(f"{path}: no extent {name!r}")
        if list(dst.shape) != e["shape"] or str(dst.dtype).replace("torch.", "") != e["dtype"]:
            raise ValueError(f"{path}: extent {name!r} is {e['dtype']}{e['shape']}, target {dst.dtype}{list(dst.shape)}")
        n = e["nbytes"]
        plen = _pad(n)
        bounce = torch.empty(plen + ALIGN, dtype=torch.uint8)
        base = (-bounce.data_ptr()) % ALIGN  # an aligned start for O_DIRECT
        buf = bounce[base: base + plen]
        for o in range(0, plen, CHUNK):
            pool.submit(path, e["offset"] + o, min(CHUNK, plen - o), buf.data_ptr() + o)
        got = pool.wait_all()
        if got < 0:
            raise OSError(-got, f"{path}: read of extent {name!r} failed")
        if got < n:
            raise ValueError(f"{path}: extent {name!r} is truncated")
        data = buf[:n]
        if verify and ext().blake3(data.numpy().tobytes()).hex() != e["blake3"]:
            raise ValueError(f"{path}: extent {name!r} failed its digest")
        _bytes_view(dst).copy_(data) if dst.is_contiguous() and dst.device.type == "cpu" else \
            dst.copy_(data.view(dst.dtype).view(dst.shape))
        total += n
    return total
