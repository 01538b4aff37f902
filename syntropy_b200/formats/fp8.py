"""Block-scaled fp8 (e4m3) weights: one f32 scale per 128x128 weight tile, value =
e4m3 * scale (the `weight_scale_inv` convention), and per-token 1x128 activation scales.
Reference: plan/rfcs/RFC-0042-quantization-and-numerical-fidelity.md §2.3."""
from __future__ import annotations

from dataclasses import dataclass

import torch

E4M3_MAX = 448.0
BLOCK = 128


def quantize_fp8_block(w: torch.Tensor, block: int = BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """w [N, K] -> (e4m3 [N, K], scale f32 [ceil(N/b), ceil(K/b)])."""
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    wp = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    wp[:N, :K] = w.float()
    t = wp.view(nb, block, kb, block)
    amax = t.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / E4M3_MAX
    q = (t / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(nb * block, kb * block)[:N, :K].contiguous(), scale.float()


def dequant_fp8_block(q: torch.Tensor, scale: torch.Tensor, block: int = BLOCK) -> torch.Tensor:
    N, K = q.shape
    s = scale.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * s


def quantize_act_fp8(x: torch.Tensor, group: int = BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token 1 x group scales: x [T, K] -> (e4m3 [T, K], scale f32 [T, K/group])."""
    T, K = x.shape
    g = x.float().view(T, K // group, group)
    s = (g.abs().amax(-1) / E4M3_MAX).clamp_min(1e-12)
    q = (g / s[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(T, K), s


@dataclass
class FP8Weight:
    """e4m3 weights with one f32 scale per 128x128 block.  On the device the bytes live in
    the mma-fragment tiled layout (``tiled``, see csrc/cuda/fp8.cu) and ``q`` is None; on the
    host ``q`` is the row-major e4m3 tensor."""
    N: int
    K: int
    q: torch.Tensor | None   # e4m3 [N, K] (host)
    scale: torch.Tensor      # f32 [ceil(N/128), ceil(K/128)]
    tiled: torch.Tensor | None = None  # uint8 [N*K] (device)

    @classmethod
    def quantize(cls, w: torch.Tensor) -> "FP8Weight":
        q, s = quantize_fp8_block(w)
        if w.is_cuda and w.shape[0] % 16 == 0 and w.shape[1] % 128 == 0:
            from .._ext import ext
            t = ext().f8_rows_to_tiled(q.view(torch.uint8).contiguous(), w.shape[0], w.shape[1])
            return cls(w.shape[0], w.shape[1], None, s.contiguous(), t)
        return cls(w.shape[0], w.shape[1], q, s)

    def rows(self) -> torch.Tensor:
        """Row-major e4m3 [N, K]."""
        if self.q is not None:
            return self.q
        from .._ext import ext
        return ext().f8_tiled_to_rows(self.tiled, self.N, self.K).view(torch.float8_e4m3fn)

    def dequant(self, dtype=torch.bfloat16) -> torch.Tensor:
        if self.tiled is not None and dtype == torch.bfloat16:
            from .._ext import ext
            return ext().f8_dequant_tiled(self.tiled, self.scale, self.N, self.K)
        return dequant_fp8_block(self.rows(), self.scale).to(dtype)

    @property
    def nbytes(self) -> int:
        return self.N * self.K + self.scale.numel() * 4
