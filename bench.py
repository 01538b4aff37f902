"""Headline benchmark: decode tok/s + p50 TTFT of the Qwen3-235B-A22B-shaped 4-bit MoE
(94 layers, hidden 4096, 64/4 heads x 128, 128 experts top-8, expert FFN 1536, vocab
151936), batch 32, prompt 1024, on N B200s, synthetic uniform-random prompts and
random-init N(0, 0.02) weights quantised to 4-bit blocks.

    python bench.py [--gpus N --steps K --warmup W]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)
    python bench.py --impl reference                       (reference arm)

`value` is whole-job decode tokens/s, device-timed with CUDA events around the decode
steps (max over ranks); `e2e` is the same metric through the public engine API
(LLMEngine.step), including the per-step host->device step-descriptor copy and the
device->host read of the sampled tokens.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s + p50 TTFT, Qwen3-235B-A22B-shape 4-bit, 1/2/4/8 B200, max over ranks"
# the other named configs (same measurement; --model selects them): batch, prompt, decode
CONFIG_DEFAULTS = {"qwen3-235b-a22b": (32, 1024, 256), "llama3-8b": (64, 2048, 256),
                   "llama3-70b": (32, 4096, 512), "deepseek-v3": (16, 2048, 256)}


def reference_arm(args):
    # The reference is a Rust workspace with no Python package, no GPU kernels and no
    # end-to-end forward; it cannot be installed as a Python package or run on this image.
    print(json.dumps({"impl": "reference", "unavailable":
                      "reference is a pre-alpha Rust workspace (no GPU kernels, no end-to-end forward, no cargo "
                      "toolchain on the box); pip install of the reference source tree fails: no setup.py/pyproject.toml"}))


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        mx = max(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="syntropy", choices=["syntropy", "reference"])
    ap.add_argument("--model", default="qwen3-235b-a22b")
    ap.add_argument("--batch", type=int, default=None, help="default: the named config's")
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--decode", type=int, default=None)
    ap.add_argument("--pp", type=int, default=1, help="dense models: pipeline stages (TP = gpus / pp)")
    ap.add_argument("--layers", type=int, default=0, help="dev only: override layer count (invalid headline)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--baseline", action="store_true", help="NCCL all-gather/reduce-scatter MoE data plane")
    ap.add_argument("--expert-cache-frac", type=float, default=None,
                    help="VRAM-resident share of each rank's experts (Qwen3 config: 0.6, rest in pinned host RAM; "
                         "others: 1.0)")
    ap.add_argument("--no-uncapped", action="store_true", help="skip the extra all-resident measurement")
    ap.add_argument("--rebalance-every", type=int, default=64,
                    help="decode steps between expert-cache adaptations (decayed-LFU swaps; 0 = never)")
    ap.add_argument("--expert-prefetch", type=int, default=1,
                    help="host-tier experts staged into VRAM during decode (1 on, 0 off: read over PCIe in place)")
    ap.add_argument("--expert-staging", default="auto", choices=["auto", "bulk", "predicted"],
                    help="bulk: DMA-copy every GPU-read host expert of each layer (best when most experts are "
                         "routed to); predicted: copy the router-predicted ones; auto: bulk when a layer's "
                         "rows are expected to reach at least half of the experts")
    ap.add_argument("--cpu-experts", type=float, default=None,
                    help="share of each layer's host-tier experts computed by host CPU threads during decode "
                         "(the rest is read over PCIe by the GPU); 0 = off (default: the share that balances the "
                         "rank's CPU workers against its host link)")
    ap.add_argument("--cpu-threads", type=int, default=None,
                    help="CPU expert threads per rank (default: the rank's share of the node's cores, less one)")
    ap.add_argument("--step-profile", action="store_true",
                    help="after the timed steps, replay one decode step through the timestamped graph variant and "
                         "report device ms per segment kind (max over ranks)")
    ap.add_argument("--no-mtp", action="store_true", help="models with an MTP head: plain decoding instead of "
                    "MTP drafting + batched verification")
    ap.add_argument("--spec", choices=["auto", "none", "ngram"], default="auto",
                    help="speculative decoding: auto = the model's MTP head when it has one; ngram = prompt-lookup "
                         "drafts of --spec-gamma tokens verified in one batched pass (one GPU, no TP/PP)")
    ap.add_argument("--spec-gamma", type=int, default=3)
    ap.add_argument("--prompt-kind", choices=["random", "repeat"], default="random",
                    help="random: uniform-random token ids (the named config); repeat: a random 64-token "
                         "pattern repeated to the prompt length (text with repetition, where prompt-lookup "
                         "drafts apply)")
    ap.add_argument("--max-prefill-tokens", type=int, default=0,
                    help="prompt tokens per prefill step (0: 8192, or every local prompt up to 32768 tokens when "
                         "host-tier experts stream through each prefill pass)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    db, dp, dd = CONFIG_DEFAULTS.get(args.model, (32, 1024, 256))
    args.batch = args.batch or db
    args.prompt = args.prompt or dp
    args.decode = args.decode or dd
    if args.expert_cache_frac is None:
        args.expert_cache_frac = 0.6 if args.model == "qwen3-235b-a22b" else 1.0

    import torch

    from syntropy_b200.models.config import get_config
    from syntropy_b200.models.transformer import prepare_weights
    from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
    from syntropy_b200.runtime.runner import ModelRunner
    from syntropy_b200 import ops

    from syntropy_b200.parallel.dist import init_distributed, max_over_ranks, shutdown

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    ctx = init_distributed(timeout_s=300)
    rank, local = ctx.rank, ctx.local_rank
    dev = ctx.device
    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.replace(n_layers=args.layers)
    ep = tp = pp = None
    tp_size = 1
    max_pos = args.prompt + max(args.decode, args.warmup + args.steps + 40) + 16
    if cfg.is_moe:
        if args.batch % world:
            raise SystemExit("global batch must divide over the GPUs")
        B = args.batch // world  # data-parallel attention: each rank serves its share of sequences
        if world > 1:
            from syntropy_b200.parallel.ep import EPGroup
            # MTP verify windows hold 2 rows per sequence: the combine slots take them all
            ep = EPGroup(ctx, cfg.n_experts, cfg.top_k, cfg.hidden, cap=B * (2 if cfg.n_mtp and not args.no_mtp else 1),
                         n_layers=cfg.n_layers, fused=not args.baseline)
        t0 = time.time()
        mw = prepare_weights(cfg, dev, seed=args.seed, max_pos=max_pos, expert_range=ep.expert_range if ep else None)
    else:
        # dense: tensor parallel over gpus/pp ranks, pipeline over pp stages; every rank of a
        # stage serves every sequence
        B = args.batch
        layer_range = None
        t0 = time.time()
        if world > 1:
            from syntropy_b200.parallel.dist import split_tp_pp
            from syntropy_b200.parallel.pp import PPGroup
            from syntropy_b200.parallel.tp import TPGroup
            if world % args.pp:
                raise SystemExit("--pp must divide the GPU count")
            tp_size = world // args.pp
            tp_ctx, pp_group, pp_ranks, stage = split_tp_pp(ctx, tp_size, args.pp)
            if args.pp > 1:
                pp = PPGroup(ctx, args.pp, stage, cfg.n_layers, group=pp_group, ranks=pp_ranks)
                layer_range = pp.layer_range
            t0 = time.time()
            mw = prepare_weights(cfg, dev, seed=args.seed, max_pos=max_pos,
                                 tp=(tp_ctx.rank, tp_size) if tp_size > 1 else None, layer_range=layer_range)
            if tp_size > 1:
                tp = TPGroup(tp_ctx, cfg.hidden, cap=B, n_layers=len(mw.layers),
                             fused=not args.baseline and cfg.weight_quant in ("q4", "bf16"),
                             vocab=cfg.vocab if cfg.weight_quant == "bf16" and (pp is None or pp.last) else 0)
        else:
            mw = prepare_weights(cfg, dev, seed=args.seed, max_pos=max_pos)
    torch.cuda.synchronize()
    t_weights = time.time() - t0
    # decode length: the config's, extended only if the requested steps need more tokens
    decode_len = max(args.decode, args.warmup + args.steps + min(args.steps, 16) + 8)
    max_len = args.prompt + decode_len
    cache = None
    if args.expert_cache_frac < 1.0 and cfg.is_moe:
        from syntropy_b200.experts.cache import ExpertCache
        cache = ExpertCache(mw.layers, args.expert_cache_frac, dev)
        if args.expert_prefetch:
            # rows one MoE layer sees per step: the global batch (every rank's rows reach an owner)
            touched = 1.0 - (1.0 - cfg.top_k / cfg.n_experts) ** args.batch
            bulk = args.expert_staging == "bulk" or (args.expert_staging == "auto" and touched >= 0.5)
            if bulk:
                cache.enable_decode_staging()
            else:
                cache.enable_decode_prefetch(cfg.n_experts)
    # TP's NCCL all-reduce baseline is captured into the decode graphs too (ranks step in lockstep)
    graphs = not ((ep is not None and not ep.fused) or pp is not None)
    use_mtp = cfg.n_mtp > 0 and mw.mtp is not None and not args.no_mtp and pp is None and tp is None and \
        args.spec == "auto"
    use_ngram = args.spec == "ngram" and pp is None and tp is None and ep is None
    # verify windows hold 1 + gamma rows per sequence (MTP: gamma 1)
    rows_per_seq = 2 if use_mtp else (1 + args.spec_gamma if use_ngram else 1)
    runner = ModelRunner(mw, max_batch=B * rows_per_seq, max_seq_len=max_len + 16 + args.spec_gamma, ep=ep, tp=tp,
                         pp=pp, use_graphs=graphs)
    runner.expert_cache = cache
    tier = None
    if cache is not None and tp is None and pp is None and (ep is None or ep.fused) and cfg.weight_quant == "q4":
        # the host CPU computes a share of each rank's cold experts; the node's cores are split
        # over its ranks (each rank's slice, less its launching thread's core)
        from syntropy_b200.experts.cpu_tier import CpuExpertTier, balanced_share, rank_cpus
        local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
        cpus, _ = rank_cpus(local, local_world)
        threads = args.cpu_threads or len(cpus)
        if args.cpu_experts is None:  # the share that balances the CPU workers and the host link
            args.cpu_experts = balanced_share(threads, local_world)
        if args.cpu_experts > 0 and threads > 0:
            tier = CpuExpertTier(cache, cfg, max_rows=runner.max_batch, cpu_share=args.cpu_experts,
                                 threads=threads, cpus=cpus, ep=ep)
    if args.cpu_experts is None:
        args.cpu_experts = 0.0
    spec = None
    if use_mtp:
        from syntropy_b200.runtime.spec import MTPDrafter, SpecConfig
        spec = SpecConfig(drafter=MTPDrafter(runner))
    elif use_ngram:
        from syntropy_b200.runtime.spec import NgramDrafter, SpecConfig
        spec = SpecConfig(drafter=NgramDrafter(), gamma=args.spec_gamma)
    # a prefill pass streams every host-tier expert of every layer over PCIe once, whatever its
    # token count: with a host tier, one pass takes all local prompts (bounded for activations)
    n_local = args.batch // world if cfg.is_moe else args.batch
    mpt = args.max_prefill_tokens or (min(32768, max(8192, n_local * args.prompt)) if cache is not None else 8192)
    eng = LLMEngine(runner, max_prefill_tokens=mpt, dist_ctx=ctx, spec=spec, rebalance_every=args.rebalance_every)
    g = torch.Generator().manual_seed(1234)
    if args.prompt_kind == "repeat":
        pats = [torch.randint(0, cfg.vocab, (64,), generator=g).tolist() for _ in range(args.batch)]
        all_prompts = [(p * (args.prompt // 64 + 1))[:args.prompt] for p in pats]
    else:
        all_prompts = [torch.randint(0, cfg.vocab, (args.prompt,), generator=g).tolist() for _ in range(args.batch)]
    prompts = all_prompts[rank::world] if cfg.is_moe else all_prompts
    # ---- warm-up (untimed): one request of the timed prompt length through prefill and two
    # decode steps, so the timed prefill meets loaded kernels, encoded tensor maps and live NCCL
    # communicators (their one-time set-up is not time to first token of a serving engine) ----
    eng.generate([all_prompts[0]], SamplingParams(max_tokens=2, temperature=0.0))
    torch.cuda.synchronize()
    # ---- prefill: TTFT of each request (all submitted at t0) ----
    ids = [eng.add_request(p, SamplingParams(max_tokens=decode_len, temperature=0.0)) for p in prompts]
    if ctx.enabled:
        import torch.distributed as dist
        dist.barrier(group=ctx.cpu_group)
    if args.step_profile and runner.is_cuda:
        runner.profile_prefill_next = True  # the first prefill pass: device ms per layer segment
    t_sub = time.perf_counter()
    if ctx.enabled:
        while _any_waiting(ctx, eng):
            eng.step()
    else:
        while eng.waiting:
            eng.step()
    torch.cuda.synchronize()
    prefill_prof = None
    if args.step_profile and runner.is_cuda:
        # every rank takes the same collective steps: a fixed list of segment kinds
        kinds = ("prefill_qkv", "prefill_attn_core", "prefill_attn", "prefill_ffn", "prefill_moe_route",
                 "prefill_moe_stage", "prefill_moe_experts", "prefill_moe", "prefill_head")
        agg = dict.fromkeys(kinds, 0.0)
        if runner._stamp_labels[-1:] == ["prefill_head"]:
            for lab, ms in runner.step_profile():
                kind = lab.split(".")[-1]
                agg[kind] = agg.get(kind, 0.0) + ms
        prefill_prof = {k: round(max_over_ranks(ctx, agg[k]), 3) for k in kinds}
        prefill_prof["tokens_in_pass"] = int(min(mpt, n_local * args.prompt))
    seqs = {s.seq_id: s for s in eng.running}
    my_ttft = [seqs[i].t_first_token - t_sub for i in ids]
    if ctx.enabled:
        import torch.distributed as dist
        gathered = [None] * world
        dist.all_gather_object(gathered, my_ttft, group=ctx.cpu_group)
        if cfg.is_moe:
            my_ttft = [x for part in gathered for x in part]
        else:  # every rank serves every sequence: a request's TTFT is its latest rank's
            my_ttft = [max(part[i] for part in gathered) for i in range(len(my_ttft))]
    ttft = sorted(my_ttft)
    p50_ttft_ms = 1e3 * ttft[len(ttft) // 2]
    # ---- decode: warm-up then timed steps ----
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    # launch count of one decode step (eager count of the captured sequence)
    n_launch = ops.count_launches(lambda: runner.decode_forward(B)) if hasattr(ops, "count_launches") else None
    # timed decode steps through the engine: device time = sum of CUDA-event-bracketed
    # graph replays; e2e = wall time of the same steps (descriptor H2D + tokens D2H)
    runner.time_events = []
    step_events = []
    tok0, acc0, dr0 = eng.stats["decode_tokens"], eng.stats.get("spec_accepted", 0), eng.stats.get("spec_drafted", 0)
    pz0 = eng.stats.get("spec_paused_steps", 0)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        te = time.perf_counter()
        for _ in range(args.steps):
            if spec is not None:  # a step is the verify pass plus the draft pass: time both
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                eng.step()
                e1.record()
                step_events.append((e0, e1))
            else:
                eng.step()
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - te
    if spec is not None:
        dev_ms = sum(a.elapsed_time(b) for a, b in step_events)
    else:
        dev_ms = sum(a.elapsed_time(b) for a, b in runner.time_events)
        assert len(runner.time_events) == args.steps
    dev_ms = max_over_ranks(ctx, dev_ms)
    e2e_s = max_over_ranks(ctx, e2e_s)
    from syntropy_b200.parallel.dist import sum_over_ranks
    timed_tokens = sum_over_ranks(ctx, float(eng.stats["decode_tokens"] - tok0))
    mtp_info = None
    if spec is not None:
        acc = sum_over_ranks(ctx, float(eng.stats["spec_accepted"] - acc0))
        drf = sum_over_ranks(ctx, float(eng.stats["spec_drafted"] - dr0))
        mtp_info = {"acceptance_rate": round(acc / max(1.0, drf), 4), "drafted": int(drf), "accepted": int(acc),
                    "tokens_per_seq_step": round(timed_tokens / (args.batch * args.steps), 4),
                    "paused_steps": int(eng.stats.get("spec_paused_steps", 0) - pz0)}
    step_prof = None
    if args.step_profile and runner.use_graphs:
        # one decode step through the timestamped graph variant (same kernels plus one
        # %globaltimer write per segment): device ms per segment kind, max over ranks
        runner.profile_next = True
        eng.step()
        agg = {}
        for lab, ms in runner.step_profile():
            kind = lab.split(".")[-1]
            agg[kind] = agg.get(kind, 0.0) + ms
        kinds = sorted(agg)
        if ctx.enabled:
            import torch.distributed as dist
            allk = [None] * world
            dist.all_gather_object(allk, agg, group=ctx.cpu_group)
            kinds = sorted({k for a in allk for k in a})
            step_prof = {k: round(max(a.get(k, 0.0) for a in allk), 4) for k in kinds}
            step_prof["rank0"] = {k: round(allk[0].get(k, 0.0), 4) for k in kinds}
        else:
            step_prof = {k: round(agg[k], 4) for k in kinds}
        # the same step as cost terms beside the planner's prediction for this configuration
        try:
            from syntropy_b200.core.plan import ParallelismMode
            from syntropy_b200.obs.spans import step_cost_record
            from syntropy_b200.planner.planner import HardwareModel, price_decode
            mode = ParallelismMode.LOCAL if world == 1 else (ParallelismMode.EP if cfg.is_moe else
                                                             ParallelismMode.INTRA_NODE_TP)
            pred = price_decode(cfg, world, args.batch, args.prompt + args.warmup + args.steps, mode,
                                args.expert_cache_frac if cfg.is_moe else 1.0, HardwareModel.from_measured(),
                                fused=not args.baseline, cpu_share=args.cpu_experts)
            rec = step_cost_record(eng.stats["decode_steps"], runner.step_profile(), pred)
            step_prof["cost_terms"] = rec.rows()
        except Exception as exc:  # noqa: BLE001  (informational)
            step_prof["cost_terms"] = f"{type(exc).__name__}: {exc}"[:200]
        step_prof["host_lockstep_ms_per_step"] = round(1e3 * eng.stats.get("lockstep_s", 0.0) /
                                                       max(1, eng.stats["decode_steps"] + eng.stats["prefill_steps"]),
                                                       4)
    status = ep.check_status() if ep is not None else 0
    tier_stats = tier.stats() if tier is not None else None
    # the timed run's expert placement (the all-resident measurement below changes it)
    placed = {"prefetch": bool(cache is not None and cache.prefetch),
              "staging": ("bulk" if cache.stage_all else "predicted" if cache.prefetch else "none")
              if cache is not None else "none",
              "host_gb": round(cache.host_bytes() / 1e9, 2) if cache is not None else 0.0,
              "weights_gb": mw.nbytes() / 1e9}
    uncapped = None
    if cache is not None and not args.no_uncapped:
        # same model and batch with every expert VRAM-resident (the cap lifted); informational,
        # so a failure here does not cost the headline line
        try:
            if tier is not None:  # nothing is left for the CPU: decode graphs without the hand-off
                tier.detach()
            runner.graphs.clear()  # and without staging copies
            cache.promote_all()
            for _ in range(2):
                eng.step()
            runner.time_events = []
            torch.cuda.synchronize()
            for _ in range(min(args.steps, 16)):
                eng.step()
            torch.cuda.synchronize()
            u_ms = max_over_ranks(ctx, sum(a.elapsed_time(b) for a, b in runner.time_events)) / len(runner.time_events)
            uncapped = {"value": round(args.batch * 1e3 / u_ms, 2), "ms_per_step": round(u_ms, 4),
                        "steps": len(runner.time_events), "expert_cache_frac": 1.0}
        except Exception as exc:  # noqa: BLE001
            uncapped = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    ms_step = dev_ms / args.steps
    # whole-job tokens/s over all ranks (with MTP: the tokens actually emitted)
    value = (timed_tokens if spec is not None else args.batch * args.steps) * 1e3 / dev_ms
    e2e_value = (timed_tokens if spec is not None else args.batch * args.steps) / e2e_s
    wq = cfg.weight_quant
    wdesc = {"q4": "4-bit block weights (32-elem, fp16 scale+min)", "bf16": "bf16 weights",
             "fp8": "fp8 e4m3 weights, 128x128 block scales"}.get(wq, wq)
    if cfg.is_moe:
        par = (f"ep{world}+dp-attention" + ("" if ep is None or ep.fused else " (nccl baseline)")) \
            if world > 1 else "single-gpu"
    else:
        par = "single-gpu" if world == 1 else (f"tp{tp_size}" + (f"xpp{args.pp}" if args.pp > 1 else "") +
                                               ("" if tp is None or tp.fused else " (nccl all-reduce baseline)"))
    metric = METRIC if args.model == "qwen3-235b-a22b" else \
        f"decode tok/s + p50 TTFT, {args.model}-shape {wq}, max over ranks"
    out = {
        "metric": metric, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": f"bf16 activations, {wdesc}",
        "data": (f"synthetic {'uniform-random' if args.prompt_kind == 'random' else 'repeated 64-token-pattern'} "
                 f"prompts, random-init N(0,0.02) weights ({wq})"),
        "p50_ttft_ms": round(p50_ttft_ms, 2),
        "config": {"model": args.model if not args.layers else f"{args.model}[layers={args.layers}] (DEV, not headline)",
                   "global_batch": args.batch, "seq_len": args.prompt, "decode_len": decode_len,
                   "max_prefill_tokens": mpt,
                   "parallelism": par,
                   "expert_cache_frac": args.expert_cache_frac if cfg.is_moe else 1.0,
                   "host_tier_gb": placed["host_gb"],
                   "expert_prefetch": placed["prefetch"],
                   "expert_staging": placed["staging"],
                   "expert_rebalance_every": args.rebalance_every if cache is not None else 0,
                   "cpu_expert_share": args.cpu_experts if tier is not None else 0.0,
                   "cpu_expert_threads": tier.threads if tier is not None else 0,  # per rank
                   "host_cores": len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else None,
                   "l2": f"inputs larger than L2 ({placed['weights_gb']:.0f} GB of weights streamed per step per rank)",
                   "weights_gb": round(placed["weights_gb"], 2), "weight_build_s": round(t_weights, 1)},
        "clocks": clk.summary(),
        "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": runner.desc.nbytes,
                "d2h_bytes_per_step": 4 * B},
        "gpu_launches": (n_launch * args.steps) if n_launch else None,
        "impl": "syntropy",
        "cpu_tier": tier_stats,
        "device_status": status,
        "all_experts_resident": uncapped,
    }
    if mtp_info is not None:
        out["mtp" if use_mtp else "spec"] = dict(mtp_info, drafter="mtp" if use_mtp else f"ngram(gamma={args.spec_gamma})")
    if step_prof is not None:
        out["step_profile_ms"] = step_prof
    if prefill_prof is not None:
        out["prefill_profile_ms"] = prefill_prof
    if rank == 0:
        print(json.dumps(out))
    runner.graphs.clear()
    if tier is not None:
        tier.close()
    shutdown(ctx)


def _any_waiting(ctx, eng) -> bool:
    import torch
    import torch.distributed as dist
    t = torch.tensor([1 if eng.waiting else 0], dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ctx.cpu_group)
    return bool(t[0])


if __name__ == "__main__":
    main()
