"""Dequantisation of GGML block formats found in GGUF checkpoints (vectorised torch, f32 out).

Layouts (the public GGML block definitions; the bytes of a file must be read as written):
  Q8_0  32 values, 34 bytes : fp16 d, 32 x int8 q                         -> d q
  Q4_0  32 values, 18 bytes : fp16 d, 16 bytes (value j low nibble, j+16 high) -> d (q - 8)
  Q4_1  32 values, 20 bytes : fp16 d, fp16 m, 16 bytes of nibbles          -> d q + m
  Q4_K 256 values, 144 bytes: fp16 d, fp16 dmin, 12 bytes of 6-bit scales and mins for
        eight 32-value sub-blocks, 128 bytes of nibbles (each 32 bytes hold two sub-blocks:
        low nibbles the first, high nibbles the second)                    -> d sc q - dmin mn
  Q6_K 256 values, 210 bytes: 128 bytes low 4 bits, 64 bytes high 2 bits, 16 int8 scales
        (one per 16 values), fp16 d                                        -> d sc (q - 32)
"""
from __future__ import annotations

import torch

BLOCKS = {"F32": (1, 4), "F16": (1, 2), "BF16": (1, 2), "Q4_0": (32, 18), "Q4_1": (32, 20), "Q8_0": (32, 34),
          "Q4_K": (256, 144), "Q6_K": (256, 210)}
GGML_TYPE = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K", 30: "BF16"}


def _f16(b: torch.Tensor) -> torch.Tensor:
    """[..., 2] uint8 -> f32"""
    return b.contiguous().view(torch.float16).float().squeeze(-1)


def _nibbles(b: torch.Tensor) -> torch.Tensor:
    """[..., 16] bytes -> [..., 32] values: low nibbles first, then high nibbles."""
    return torch.cat([b & 15, b >> 4], -1).float()


def dequant_q8_0(raw: torch.Tensor) -> torch.Tensor:
    b = raw.view(-1, 34)
    return (_f16(b[:, :2])[:, None] * b[:, 2:].view(torch.int8).float()).reshape(-1)


def dequant_q4_0(raw: torch.Tensor) -> torch.Tensor:
    b = raw.view(-1, 18)
    return (_f16(b[:, :2])[:, None] * (_nibbles(b[:, 2:]) - 8)).reshape(-1)


def dequant_q4_1(raw: torch.Tensor) -> torch.Tensor:
    b = raw.view(-1, 20)
    return (_f16(b[:, :2])[:, None] * _nibbles(b[:, 4:]) + _f16(b[:, 2:4])[:, None]).reshape(-1)


def _k_scales(s: torch.Tensor):
    """12 packed bytes -> (scales [n, 8], mins [n, 8]) of six bits each."""
    s = s.to(torch.int32)
    lo_sc, lo_mn = s[:, 0:4] & 63, s[:, 4:8] & 63
    hi_sc = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    hi_mn = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return torch.cat([lo_sc, hi_sc], 1).float(), torch.cat([lo_mn, hi_mn], 1).float()


def dequant_q4_k(raw: torch.Tensor) -> torch.Tensor:
    b = raw.view(-1, 144)
    d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    sc, mn = _k_scales(b[:, 4:16])
    qs = b[:, 16:].reshape(-1, 4, 32)                              # four pairs of sub-blocks
    q = torch.stack([qs & 15, qs >> 4], 2).reshape(-1, 8, 32).float()  # sub-block j = pair j//2, nibble j%2
    return (d[:, None, None] * sc[:, :, None] * q - dmin[:, None, None] * mn[:, :, None]).reshape(-1)


def dequant_q6_k(raw: torch.Tensor) -> torch.Tensor:
    b = raw.view(-1, 210)
    ql, qh = b[:, 0:128].reshape(-1, 2, 64).to(torch.int32), b[:, 128:192].reshape(-1, 2, 32).to(torch.int32)
    sc = b[:, 192:208].view(torch.int8).float().reshape(-1, 2, 8)
    d = _f16(b[:, 208:210])
    lo, hi = ql[:, :, :32], ql[:, :, 32:]
    q = torch.stack([(lo & 15) | ((qh & 3) << 4), (hi & 15) | (((qh >> 2) & 3) << 4),
                     (lo >> 4) | (((qh >> 4) & 3) << 4), (hi >> 4) | (((qh >> 6) & 3) << 4)], 2)  # [n, 2, 4, 32]
    q = (q - 32).float()
    # value l of group g (32 values) in half h uses scale 8h + 2g + l // 16
    s = sc.reshape(-1, 2, 4, 2)                                   # [n, half, group, l // 16]
    s = s.repeat_interleave(16, dim=3)                            # [n, 2, 4, 32]
    return (d[:, None, None, None] * s * q).reshape(-1)


DEQUANT = {"Q8_0": dequant_q8_0, "Q4_0": dequant_q4_0, "Q4_1": dequant_q4_1, "Q4_K": dequant_q4_k,
           "Q6_K": dequant_q6_k}
