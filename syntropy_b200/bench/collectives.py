"""Prefill all-reduce on N GPUs: the ordered two-shot kernel pair over NVLink peer memory
against NCCL's all-reduce (+ the residual add), for f32 messages of T x H.

Run: python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1
     --master-port P -m syntropy_b200.bench.collectives
Device time from CUDA events over 10 iterations after 3 warm-ups, max over ranks; the
roofline is the bytes that must cross NVLink per direction ((N-1)/N of the message for a
reduce-scatter + all-gather) at the measured 770 GB/s peer bandwidth.
"""
from __future__ import annotations

import json

import torch
import torch.distributed as dist

from ..parallel.dist import init_distributed, shutdown
from ..parallel.tp import TPGroup

PEER_GBS = 770.0


def _time(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3  # us


def main():
    ctx = init_distributed(timeout_s=60)
    dev, N = ctx.device, ctx.world
    H = 8192
    tp = TPGroup(ctx, H, cap=64, n_layers=1, fused=True)
    for T in (128, 512, 2048):
        if T > tp.prefill_rows:
            continue
        x = torch.zeros(T, H, device=dev)
        tp.part_view(T).normal_()
        part = torch.randn(T, H, device=dev)

        def twoshot():
            tp.twoshot_add(x)

        def nccl():
            dist.all_reduce(part, group=ctx.group)
            x.add_(part)

        dist.barrier(group=ctx.cpu_group)
        t2 = _time(twoshot)
        dist.barrier(group=ctx.cpu_group)
        tn = _time(nccl)
        ts = torch.tensor([t2, tn], device=dev)
        dist.all_reduce(ts, op=dist.ReduceOp.MAX, group=ctx.group)
        t2, tn = ts.tolist()
        msg = T * H * 4
        roof_us = (N - 1) / N * msg / (PEER_GBS * 1e9) * 1e6
        if ctx.rank == 0:
            print(json.dumps({"collective": "prefill_allreduce", "n_gpus": N, "rows": T, "hidden": H,
                              "bytes": msg, "twoshot_us": round(t2, 1), "nccl_us": round(tn, 1),
                              "roofline_us": round(roof_us, 1), "twoshot_frac_of_roofline": round(roof_us / t2, 3),
                              "status": tp.check_status()}), flush=True)
    dist.barrier(group=ctx.cpu_group)
    shutdown(ctx)


if __name__ == "__main__":
    main()
