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


def numa_cpus(gpu_index: int, nvml=None) -> list[int] | None:
    """CPUs of the NUMA node closest to GPU `gpu_index` (NVML CPU-affinity bitmask), or None
    when NVML is unavailable.  `nvml` can be a stand-in module with the same three calls."""
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        h = nvml.nvmlDeviceGetHandleByIndex(gpu_index)
        words = nvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
    except Exception:
        return None
    cpus = [w * 64 + b for w, m in enumerate(words) for b in range(64) if (int(m) >> b) & 1]
    return cpus or None


def bind_to_gpu_numa(gpu_index: int, nvml=None) -> bool:
    """Pins this process to the CPUs next to its GPU, so pinned host memory it allocates
    afterwards (the cold expert tier, staging buffers) lands on the GPU-local NUMA node and
    host-to-GPU reads do not cross the socket interconnect.  Off with SYN_NUMA_BIND=0."""
    if os.environ.get("SYN_NUMA_BIND", "1") != "1" or not hasattr(os, "sched_setaffinity"):
        return False
    cpus = numa_cpus(gpu_index, nvml)
    if not cpus:
        return False
    allowed = os.sched_getaffinity(0)
    pick = [c for c in cpus if c in allowed]
    if not pick:
        return False
    os.sched_setaffinity(0, pick)
    return True


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> DistContext:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
        bind_to_gpu_numa(torch.cuda.current_device())
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


def split_tp_pp(ctx: DistContext, tp: int, pp: int):
    """TP x PP layout over the world: global rank = stage * tp + tp_index.  Returns
    (tp_ctx, pp_group, pp_ranks, stage): tp_ctx is a DistContext over this rank's TP group
    (its stage), pp_group/pp_ranks link this TP index across the stages.  Every rank creates
    every group in the same order (a torch.distributed requirement)."""
    assert tp * pp == ctx.world, "tp * pp must equal the world size"
    stage, t = divmod(ctx.rank, tp)
    nccl = dist.get_backend(ctx.group) == "nccl"
    tp_ctx = pp_group = pp_ranks = None
    for s in range(pp):
        ranks = [s * tp + i for i in range(tp)]
        g = dist.new_group(ranks)
        cg = dist.new_group(ranks, backend="gloo") if nccl else g
        if s == stage:
            tp_ctx = DistContext(t, tp, ctx.local_rank, ctx.device, g, cg)
    for i in range(tp):
        ranks = [s * tp + i for s in range(pp)]
        g = dist.new_group(ranks)
        if i == t:
            pp_group, pp_ranks = g, ranks
    return tp_ctx, pp_group, pp_ranks, stage


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
