"""The host CPU expert pool alone, at Qwen3-235B-A22B layer size: the pool owns `owned` experts
of each layer (4-bit gate/up 3072 x 4096 and down 4096 x 1536, synthetic bytes), batch-32 rows
are routed top-8 over 128 experts, and each layer is released through the mailbox exactly as
the GPU hand-off kernel does it (rows, routing CSR, go word); the time is wall time from the go
word to the done word, median over the layers.  No GPU is used.

Run: python -m syntropy_b200.bench.cpu_pool [--layers 3] [--threads 14] [--owned 36]
Environment overrides of the pool (SYN_CPU_TASK_TILES, SYN_CPU_PREFETCH, SYN_CPU_GEMV_MODE)
apply, for comparisons.  The weight buffers are pageable host memory (the engine's tier is
pinned), so absolute rates are lower than in the engine; compare settings with each other.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch

from .._ext import ext


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=3)
    ap.add_argument("--threads", type=int, default=None, help="workers (default: allowed cores - 2)")
    ap.add_argument("--owned", type=int, default=36, help="CPU-owned experts per layer")
    ap.add_argument("--rows", type=int, default=32)
    ap.add_argument("--repeats", type=int, default=3)
    args = ap.parse_args()
    E, k, H, I, R = 128, 8, 4096, 1536, args.rows
    allowed = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(os.cpu_count()))
    threads = args.threads or max(1, len(allowed) - 2)
    cpus = allowed[1:1 + threads]
    torch.manual_seed(0)
    o_off, o_idx, o_pw, o_h, _, _, nbytes = ext().cpu_mailbox_bytes(E, k, R, H)
    mb = torch.zeros(nbytes, dtype=torch.uint8)
    w32 = mb.view(torch.int32)
    tier = ext().CpuExpertTier(args.layers, E, H, I, k, R, mb.data_ptr(), cpus, threads, -1)
    keep, per_layer = [], 0
    for L in range(args.layers):
        for e in torch.randperm(E)[:args.owned].tolist():
            qg = torch.randint(0, 256, (I * H,), dtype=torch.uint8)            # 2I x H nibbles
            sg = torch.full((2 * I * H // 16,), 0x2000, dtype=torch.int16)     # (d, m) per 32
            qd = torch.randint(0, 256, (H * I // 2,), dtype=torch.uint8)
            sd = torch.full((H * I // 16,), 0x2000, dtype=torch.int16)
            keep += [qg, sg, qd, sd]
            if L == 0:
                per_layer += qg.numel() + 2 * sg.numel() + qd.numel() + 2 * sd.numel()
            tier.set_expert(L, e, qg.data_ptr(), sg.data_ptr(), qd.data_ptr(), sd.data_ptr())
    tier.start()
    seq, times = 0, []
    try:
        for it in range(args.repeats + 1):
            for L in range(args.layers):
                ids = torch.stack([torch.randperm(E)[:k] for _ in range(R)])
                pairs = sorted((int(ids[t, j]), t) for t in range(R) for j in range(k))
                cnt = torch.bincount(torch.tensor([p[0] for p in pairs]), minlength=E)
                off = torch.cat([torch.zeros(1, dtype=torch.int64), cnt.cumsum(0)]).int()
                mb[o_off:o_off + 4 * (E + 1)].view(torch.int32).copy_(off)
                mb[o_idx:o_idx + 4 * R * k].view(torch.int32).copy_(torch.tensor([t for _, t in pairs]).int())
                mb[o_pw:o_pw + 4 * R * k].view(torch.float32).fill_(1.0 / k)
                mb[o_h:o_h + 2 * R * H].view(torch.bfloat16).copy_(torch.randn(R * H).bfloat16())
                seq += 1
                w32[1], w32[2] = L, R
                t0 = time.perf_counter()
                w32[0] = seq
                while int(w32[16]) != seq:
                    if time.perf_counter() - t0 > 30:
                        raise RuntimeError("the CPU pool did not answer")
                if it > 0:  # the first pass over the layers warms up
                    times.append(time.perf_counter() - t0)
        st = tier.stats()
    finally:
        tier.stop()
    t = sorted(times)[len(times) // 2]
    print(json.dumps({"bench": "cpu_expert_pool", "threads": threads, "mode": st["mode"],
                      "owned_bytes_per_layer": per_layer, "layer_ms": round(t * 1e3, 3),
                      "gbs_owned": round(per_layer / t / 1e9, 1), "gbs_per_thread": round(per_layer / t / 1e9 / threads, 2),
                      "task_tiles": os.environ.get("SYN_CPU_TASK_TILES", "4,8"),
                      "prefetch": os.environ.get("SYN_CPU_PREFETCH", "16")}))


if __name__ == "__main__":
    main()
