"""Collective helpers over torch.distributed that work on NCCL (device tensors, CUDA-graph
capturable) and on gloo (CPU ranks in tests), where some tensor APIs are missing."""
from __future__ import annotations

import torch
import torch.distributed as dist


def _is_nccl(group) -> bool:
    try:
        return dist.get_backend(group) == "nccl"
    except Exception:
        return False


def all_gather_rows(out: torch.Tensor, inp: torch.Tensor, group) -> torch.Tensor:
    """out[r*T:(r+1)*T] = inp of rank r."""
    if _is_nccl(group):
        dist.all_gather_into_tensor(out, inp, group=group)
        return out
    n = dist.get_world_size(group)
    parts = list(out.chunk(n, 0))
    tmp = [torch.empty_like(inp) for _ in range(n)]
    dist.all_gather(tmp, inp.contiguous(), group=group)
    for p, t in zip(parts, tmp):
        p.copy_(t)
    return out


def reduce_scatter_rows(out: torch.Tensor, inp: torch.Tensor, group) -> torch.Tensor:
    """out = sum over ranks of inp[rank*T:(rank+1)*T]."""
    if _is_nccl(group):
        dist.reduce_scatter_tensor(out, inp, group=group)
        return out
    full = inp.clone()
    dist.all_reduce(full, group=group)
    r = dist.get_rank(group)
    n = dist.get_world_size(group)
    out.copy_(full.chunk(n, 0)[r])
    return out


def all_reduce_sum(t: torch.Tensor, group) -> torch.Tensor:
    dist.all_reduce(t, group=group)
    return t
