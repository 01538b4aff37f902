"""Step profiling harness: builds a model of a named shape, prefills a batch, then runs
decode steps between cudaProfilerStart/Stop so that ``ncu --profile-from-start off`` sees
only the decode kernels.  ``--kernel-table`` instead prints the device time per kernel
name (CUPTI through torch.profiler) for the prefill of the batch and for the decode steps:
shares for finding the hot spots, not benchmark numbers.

    python -m syntropy_b200.bench.profile_decode --model qwen3-235b-a22b --layers 4 \
        --batch 32 --prompt 1024 --steps 2 [--eager] [--kernel-table]
"""
from __future__ import annotations

import argparse
import json
import time

import torch

from ..models.config import get_config
from ..models.transformer import prepare_weights
from ..runtime.engine import LLMEngine, SamplingParams
from ..runtime.runner import ModelRunner


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-235b-a22b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--eager", action="store_true", help="no CUDA graph (one launch per op)")
    ap.add_argument("--expert-cache-frac", type=float, default=1.0)
    ap.add_argument("--cpu-experts", type=float, default=0.0,
                    help="share of the host-tier experts computed by host CPU threads (with a VRAM cap)")
    ap.add_argument("--kernel-table", action="store_true", help="per-kernel device time of prefill and decode")
    ap.add_argument("--step-profile", action="store_true",
                    help="one decode step through the timestamped graph variant: device ms per segment")
    ap.add_argument("--top", type=int, default=25)
    args = ap.parse_args()
    dev = torch.device("cuda:0")
    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.replace(n_layers=args.layers)
    mw = prepare_weights(cfg, dev, seed=0, max_pos=args.prompt + 64)
    runner = ModelRunner(mw, max_batch=args.batch, max_seq_len=args.prompt + 64, use_graphs=not args.eager)
    if args.expert_cache_frac < 1.0:
        from ..experts.cache import ExpertCache
        runner.expert_cache = ExpertCache(mw.layers, args.expert_cache_frac, dev)
        if args.cpu_experts > 0:
            from ..experts.cpu_tier import CpuExpertTier
            CpuExpertTier(runner.expert_cache, cfg, max_rows=runner.max_batch, cpu_share=args.cpu_experts)
    eng = LLMEngine(runner)
    g = torch.Generator().manual_seed(0)
    for _ in range(args.batch):
        eng.add_request(torch.randint(0, cfg.vocab, (args.prompt,), generator=g).tolist(),
                        SamplingParams(max_tokens=args.warmup + args.steps + 4))
    if args.kernel_table:
        _kernel_table(eng, args)
        return
    while eng.waiting:
        eng.step()
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    if args.step_profile:
        runner.profile_next = True
        eng.step()
        prof = runner.step_profile()
        agg = {}
        for lab, ms in prof:
            kind = lab.split(".")[-1]
            agg[kind] = agg.get(kind, 0.0) + ms
        print(json.dumps({"segments_ms": {k: round(v, 4) for k, v in agg.items()},
                          "total_ms": round(sum(ms for _, ms in prof), 4)}))
        return
    runner.time_events = []
    torch.cuda.profiler.start()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    wall = time.perf_counter() - t0
    dev_ms = sum(a.elapsed_time(b) for a, b in runner.time_events) / args.steps
    print(json.dumps({"model": cfg.name, "layers": cfg.n_layers, "batch": args.batch, "ms_per_step": dev_ms,
                      "wall_ms_per_step": 1e3 * wall / args.steps}))


def _table(prof, top: int) -> list[dict]:
    rows = {}
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        r = rows.setdefault(ev.name, [0, 0.0])
        r[0] += 1
        r[1] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
    total = sum(v[1] for v in rows.values()) or 1.0
    out = [{"kernel": k[:90], "calls": v[0], "ms": round(v[1] / 1e3, 3), "share": round(v[1] / total, 4)}
           for k, v in sorted(rows.items(), key=lambda kv: -kv[1][1])[:top]]
    out.append({"kernel": "TOTAL", "ms": round(total / 1e3, 3)})
    return out


def _kernel_table(eng, args):
    from torch.profiler import ProfilerActivity, profile
    # warm-up prefill + decode so that one-time set-up is outside the profiled region
    while eng.waiting:
        eng.step()
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    runner = eng.runner
    cfg = runner.cfg
    g = torch.Generator().manual_seed(1)
    for s in list(eng.running):
        eng.abort(s.seq_id)
    for _ in range(args.batch):
        eng.add_request(torch.randint(0, cfg.vocab, (args.prompt,), generator=g).tolist(),
                        SamplingParams(max_tokens=args.steps + 4))
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        t0 = time.perf_counter()
        while eng.waiting:
            eng.step()
        torch.cuda.synchronize()
        t_pre = time.perf_counter() - t0
    print(json.dumps({"phase": "prefill", "tokens": args.batch * args.prompt, "wall_ms": round(1e3 * t_pre, 2),
                      "table": _table(prof, args.top)}))
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            eng.step()
        torch.cuda.synchronize()
    print(json.dumps({"phase": "decode", "steps": args.steps, "table": _table(prof, args.top)}))


if __name__ == "__main__":
    main()
