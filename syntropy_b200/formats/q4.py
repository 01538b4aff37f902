"""4-bit block-quantised weights: 32-element blocks along K, fp16 scale d and min m,
value = d * q + m (q in 0..15).  Byte layouts are defined in csrc/include/syn/q4.h:
the row-block interchange layout (GGUF Q4_1 blocks, 20 bytes per block) used in files,
and the tiled device layout the kernels read.

Reference: plan/rfcs/RFC-0042-quantization-and-numerical-fidelity.md §2.1 (Q4_1 row).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .._ext import ext

BLOCK = 32
ROW_BLOCK_BYTES = 20


def quantize_rows_ref(w: torch.Tensor) -> torch.Tensor:
    """Pure-torch quantiser (f32 [N, K] -> uint8 rows); same rule as the C++/CUDA ones."""
    N, K = w.shape
    b = w.float().reshape(N, K // BLOCK, BLOCK)
    mn = b.amin(-1)
    mx = b.amax(-1)
    d16 = ((mx - mn) / 15.0).to(torch.float16)
    m16 = mn.to(torch.float16)
    d = d16.float()[..., None]
    m = m16.float()[..., None]
    q = torch.where(d == 0, torch.zeros_like(b), torch.clamp(torch.round((b - m) / d), 0, 15))
    q = q.to(torch.uint8)
    qs = q[..., :16] | (q[..., 16:] << 4)
    out = torch.empty(N, K // BLOCK, ROW_BLOCK_BYTES, dtype=torch.uint8)
    out[..., 0:2] = d16.view(torch.uint8).reshape(N, K // BLOCK, 2)
    out[..., 2:4] = m16.view(torch.uint8).reshape(N, K // BLOCK, 2)
    out[..., 4:] = qs
    return out.reshape(-1)


def dequant_rows_ref(rows: torch.Tensor, N: int, K: int) -> torch.Tensor:
    r = rows.reshape(N, K // BLOCK, ROW_BLOCK_BYTES)
    d = r[..., 0:2].contiguous().view(torch.float16).float()
    m = r[..., 2:4].contiguous().view(torch.float16).float()
    qs = r[..., 4:].to(torch.int32)
    q = torch.cat([qs & 15, qs >> 4], dim=-1).float()
    return (d * q + m).reshape(N, K)


@dataclass
class Q4Weight:
    """A [N, K] matrix in the tiled device layout (or row blocks on CPU)."""

    N: int
    K: int
    qw: torch.Tensor  # int32 [N*K/8] tiled (device)
    sm: torch.Tensor  # fp16 [N*K/16] tiled (device)

    @classmethod
    def quantize(cls, w: torch.Tensor) -> "Q4Weight":
        N, K = w.shape
        qw, sm = ext().q4_quantize(w.contiguous())
        return cls(N, K, qw, sm)

    @classmethod
    def from_rows(cls, rows: torch.Tensor, N: int, K: int) -> "Q4Weight":
        if rows.is_cuda:
            qw, sm = ext().q4_rows_to_tiled(rows.contiguous(), N, K)
        else:
            qw, sm = ext().q4_rows_to_tiled_cpu(rows.contiguous(), N, K)
        return cls(N, K, qw, sm)

    def to_rows(self) -> torch.Tensor:
        return ext().q4_tiled_to_rows(self.qw, self.sm, self.N, self.K)

    def dequant(self) -> torch.Tensor:
        return ext().q4t_dequant(self.qw, self.sm, self.N, self.K)

    @property
    def nbytes(self) -> int:
        return self.qw.numel() * 4 + self.sm.numel() * 2


def q4_bytes(N: int, K: int) -> int:
    return N * K // BLOCK * ROW_BLOCK_BYTES
