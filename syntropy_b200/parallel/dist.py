"""Process-group bring-up: one process per GPU, NCCL for device collectives, gloo for
host-side control (step decisions, object exchange).  Rendezvous on 127.0.0.1."""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistContext:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    group: object = None       # device collectives (nccl on GPU, gloo on CPU)
    cpu_group: object = None   # host control plane (gloo)

    @property
    def enabled(self) -> bool:
        return self.world > 1


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> DistContext:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    if world == 1:
        return DistContext(0, 1, 0, device)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    backend = backend or ("nccl" if use_cuda else "gloo")
    to = datetime.timedelta(seconds=timeout_s)
    if not dist.is_initialized():
        kw = {"device_id": device} if backend == "nccl" else {}
        dist.init_process_group(backend=backend, rank=rank, world_size=world, timeout=to, **kw)
    group = dist.group.WORLD
    cpu_group = dist.new_group(backend="gloo", timeout=to) if backend == "nccl" else group
    return DistContext(rank, world, local, device, group, cpu_group)


def max_over_ranks(ctx: DistContext, value: float) -> float:
    if not ctx.enabled:
        return value
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctx.cpu_group)
    return float(t.item())


def sum_over_ranks(ctx: DistContext, value: float) -> float:
    if not ctx.enabled:
        return value
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=ctx.cpu_group)
    return float(t.item())


def shutdown(ctx: DistContext):
    if ctx.enabled and dist.is_initialized():
        dist.destroy_process_group()
