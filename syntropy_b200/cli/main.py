"""syntropy_b200 CLI: serve, run, plan, bench, probe, doctor, config, version."""
from __future__ import annotations

import argparse
import json
import os
import sys


def _engine_from_config(cfg, device: str):
    import torch

    from ..models.config import get_config
    from ..models.transformer import prepare_weights
    from ..runtime.engine import LLMEngine
    from ..runtime.runner import ModelRunner
    dev = torch.device(device)
    from .. import ops
    if not cfg.feature("tcgen05_attention"):
        ops.core._ATTN_TC[0] = "0"   # the mma.sync prefill attention kernel
    if not cfg.feature("tcgen05_bf16_gemm"):
        ops.core._BF16_TC[0] = "0"   # the library GEMM for bf16 weights
    sd = None
    if cfg.model.path and cfg.model.path.endswith(".gguf"):
        from ..models.hf import load_gguf  # a llama.cpp GGUF file (blocks dequantised, then requantised)
        mcfg, sd = load_gguf(cfg.model.path, weight_quant=cfg.model.quant or ("bf16" if dev.type == "cuda" else "fp32"),
                             lazy=True)
    elif cfg.model.path and os.path.exists(os.path.join(cfg.model.path, "config.json")):
        from ..models.hf import load_hf_lazy  # a Hugging Face checkpoint directory, read tensor by tensor
        mcfg, sd = load_hf_lazy(cfg.model.path,
                                weight_quant=cfg.model.quant or ("bf16" if dev.type == "cuda" else "fp32"))
    else:
        mcfg = get_config(cfg.model.name)
        if cfg.model.quant:
            mcfg = mcfg.replace(weight_quant=cfg.model.quant)
        if cfg.model.path:
            from ..formats.safetensors import load_state_dict
            sd = load_state_dict(cfg.model.path)
    mw = prepare_weights(mcfg, dev, seed=cfg.model.seed, state_dict=sd, max_pos=cfg.model.max_seq_len + 16)
    cache = None
    if cfg.tier.expert_cache_frac < 1.0 and mcfg.is_moe and dev.type == "cuda":
        from ..experts.cache import ExpertCache
        cache = ExpertCache(mw.layers, cfg.tier.expert_cache_frac, dev)
        if cfg.tier.expert_prefetch and cfg.feature("expert_prefetch"):
            cache.enable_decode_prefetch(mcfg.n_experts)  # router-predicted prefetch of host experts
    kv_budget = cfg.tier.kv_budget or None
    runner = ModelRunner(mw, max_batch=cfg.sched.max_batch, max_seq_len=cfg.model.max_seq_len,
                         use_graphs=cfg.sched.cuda_graphs and cfg.feature("cuda_graph"), kv_budget_bytes=kv_budget)
    runner.expert_cache = cache
    if cache is not None and cfg.tier.cpu_expert_share > 0 and cfg.feature("cpu_tier"):
        from ..experts.cpu_tier import CpuExpertTier
        CpuExpertTier(cache, mcfg, max_rows=runner.max_batch, cpu_share=cfg.tier.cpu_expert_share,
                      threads=cfg.tier.cpu_threads or None, timeout_s=cfg.kernels.spin_timeout,
                      mode=cfg.kernels.cpu_gemv_mode)
    spec = _spec_from_config(cfg, mcfg, runner, dev) if cfg.feature("speculative") else None
    chunk = cfg.sched.chunk_tokens or None
    return LLMEngine(runner, max_prefill_tokens=cfg.sched.max_prefill_tokens, rebalance_every=cfg.tier.rebalance_every,
                     spec=spec, chunk_tokens=chunk if spec is None else None,
                     kv_host_bytes=cfg.tier.kv_host_budget or None,
                     kv_spill_dir=cfg.tier.kv_spill_dir or None), mcfg


def _spec_from_config(cfg, mcfg, runner, dev):
    """Speculative decoding from the `spec` section (none | ngram | mtp | draft)."""
    from ..runtime.spec import DraftModelDrafter, MTPDrafter, NgramDrafter, SpecConfig
    kind = cfg.spec.drafter
    if kind == "none":
        return None
    if kind == "ngram":
        return SpecConfig(gamma=cfg.spec.gamma, drafter=NgramDrafter())
    if kind == "mtp":
        if not mcfg.n_mtp:
            raise ValueError(f"spec.drafter = mtp: {mcfg.name} has no MTP head")
        return SpecConfig(drafter=MTPDrafter(runner))
    from ..models.config import get_config
    from ..models.transformer import prepare_weights
    from ..runtime.runner import ModelRunner
    dcfg = get_config(cfg.spec.draft_model)
    if dcfg.vocab != mcfg.vocab:
        raise ValueError(f"draft model {dcfg.name} has vocabulary {dcfg.vocab}, the target {mcfg.vocab}")
    dmw = prepare_weights(dcfg, dev, seed=cfg.model.seed, max_pos=cfg.model.max_seq_len + 16 + cfg.spec.gamma)
    drunner = ModelRunner(dmw, max_batch=cfg.sched.max_batch, max_seq_len=cfg.model.max_seq_len + cfg.spec.gamma + 1,
                          use_graphs=False)
    return SpecConfig(gamma=cfg.spec.gamma, drafter=DraftModelDrafter(drunner, temperature=cfg.spec.draft_temperature))


def cmd_version(args, cfg):
    from .. import __version__
    print(json.dumps({"version": __version__, "arch": "sm_100a"}))


def cmd_config(args, cfg):
    """`config` shows the resolved values and their origins; `config get KEY`, `config set KEY
    VALUE --file F` (a format-preserving edit of the TOML file)."""
    action = getattr(args, "action", None)
    if action == "get":
        sec, _, key = args.key.rpartition(".")
        print(json.dumps({"key": args.key, "value": getattr(getattr(cfg, sec), key),
                          "origin": cfg.origin.get(args.key, "default")}))
    elif action == "set":
        from ..config.write import set_value
        path = args.file or args.config or "syntropy.toml"
        set_value(path, args.key, args.value)
        print(json.dumps({"file": path, "key": args.key, "value": args.value}))
    else:
        print(json.dumps({"config": cfg.to_dict(), "origin": cfg.origin}, indent=2))


def cmd_plan(args, cfg):
    from ..models.config import get_config
    from ..planner import HardwareModel, plan_placement
    hw = None
    if getattr(args, "probe", None):  # price from a probe report of this machine
        with open(args.probe) as f:
            hw = HardwareModel.from_probe(json.load(f))
    p = plan_placement(get_config(cfg.model.name), args.gpus, args.batch, args.ctx,
                       cache_frac=args.expert_cache_frac, fused=cfg.parallel.fused_collectives, hw=hw)
    print(p.describe() if args.explain else json.dumps({"mode": p.stages[0].mode.value,
                                                        "expert_cache_frac": p.expert_cache_frac,
                                                        "cpu_expert_share": round(p.cpu_expert_share, 3),
                                                        "predicted_step_ms": p.predicted_step_ms}))


def cmd_run(args, cfg):
    from ..runtime.engine import SamplingParams
    from ..text.tokenizer import load_tokenizer
    eng, mcfg = _engine_from_config(cfg, args.device)
    tok = load_tokenizer(cfg.model.path or None, mcfg.vocab)
    ids = [int(x) for x in args.tokens.split(",")] if args.tokens else tok.encode(args.prompt)
    eng.set_tokenizer(tok)
    stop = tuple(getattr(tok, "stop_token_ids", ()) or ())  # a checkpoint's end-of-sequence / end-of-turn ids
    constraint = {"type": "json"} if getattr(args, "json", False) else (
        {"choices": args.choices.split("|")} if getattr(args, "choices", None) else None)
    out = eng.generate([ids], SamplingParams(max_tokens=args.max_tokens, temperature=args.temperature,
                                             seed=args.seed, constraint=constraint, stop_token_ids=stop))[0]
    print(json.dumps({"tokens": out, "text": tok.decode(out)}))


def cmd_chat(args, cfg):
    """Interactive chat over the engine: each line typed is a user turn, the reply is generated
    with the model's chat template and stop tokens and printed; the conversation is kept as
    context.  `/exit` (or end of input) ends it, `/reset` starts a new conversation."""
    from ..runtime.engine import SamplingParams
    from ..text.chat import chat_ids
    from ..text.tokenizer import load_tokenizer
    eng, mcfg = _engine_from_config(cfg, args.device)
    tok = load_tokenizer(cfg.model.path or None, mcfg.vocab)
    eng.set_tokenizer(tok)
    stop = tuple(getattr(tok, "stop_token_ids", ()) or ())
    src = open(args.input) if args.input else sys.stdin
    messages = []
    try:
        for line in src:
            text = line.rstrip("\n")
            if text == "/exit":
                break
            if text == "/reset":
                messages = []
                continue
            if not text:
                continue
            messages.append({"role": "user", "content": text})
            ids = chat_ids(tok, messages, args.system)
            out = eng.generate([ids], SamplingParams(max_tokens=args.max_tokens, temperature=args.temperature,
                                                     seed=args.seed, stop_token_ids=stop))[0]
            reply = tok.decode([t for t in out if t not in stop])
            messages.append({"role": "assistant", "content": reply})
            print(json.dumps({"reply": reply, "tokens": len(out)}) if args.json else reply, flush=True)
    finally:
        if src is not sys.stdin:
            src.close()


def cmd_ls(args, cfg):
    """Models in the local store (name, id, files, bytes); --verify re-checks every file's digest."""
    from ..store.local import ModelStore
    st = ModelStore(args.store)
    for name in st.list():
        e = st.index[name]
        line = {"name": name, "model_id": e["model_id"], "files": len(e["files"]),
                "bytes": sum(f["bytes"] for f in e["files"].values())}
        if args.verify:
            line["damaged"] = st.verify(name)
        print(json.dumps(line))


def runner_table(shm_dir: str = "/dev/shm") -> list[dict]:
    """Runner processes on this host, from the shared-memory status regions their daemons
    created (`/syn-runner-<daemon pid>-<id>`): pid, lifecycle state, seconds since the last
    heartbeat, step counter, pending work, error code, and whether the pid is alive."""
    import time

    from .._ext import ext
    from ..net.ipc import HEADER_BYTES, StatusHeader
    rows = []
    try:
        names = sorted(n for n in os.listdir(shm_dir) if n.startswith("syn-runner-"))
    except OSError:
        return rows
    now = time.monotonic_ns()
    for n in names:
        try:
            reg = ext().ShmRegion("/" + n, HEADER_BYTES, False)
        except RuntimeError:
            continue  # gone since the listing, or not ours to read
        h = StatusHeader(reg.address())
        if not h.valid():
            continue
        pid = h.pid
        try:
            os.kill(pid, 0)
            alive = pid > 0
        except OSError:
            alive = False
        hb = h.heartbeat_ns
        rows.append({"region": "/" + n, "daemon_pid": int(n.split("-")[2]), "pid": pid, "state": h.state,
                     "heartbeat_age_s": round((now - hb) / 1e9, 3) if hb else None, "step": h.step,
                     "pending": h.pending, "error": h.error, "alive": alive})
        del h, reg
    return rows


def cmd_ps(args, cfg):
    """Runner processes on this host (one JSON line each)."""
    for r in runner_table():
        print(json.dumps(r))


def cmd_serve(args, cfg):
    from ..daemon.bundle import install_crash_handler
    from ..obs.log import install as install_log_suppression
    install_crash_handler(os.path.expanduser("~/.cache/syntropy_b200/crashes"))
    install_log_suppression()
    import uvicorn

    from ..api import build_app
    from ..runtime.async_engine import AsyncEngine
    from ..text.tokenizer import load_tokenizer
    eng, mcfg = _engine_from_config(cfg, args.device)
    aeng = AsyncEngine(eng)
    app = build_app(aeng, load_tokenizer(cfg.model.path or None, mcfg.vocab), model_id=cfg.api.model_id,
                    bench_api=cfg.debug.bench_api)
    uvicorn.run(app, host=cfg.api.host, port=cfg.api.port, log_level="warning")


def cmd_probe(args, cfg):
    from ..probe import probe_all
    rep = probe_all(quick=not args.full)
    if getattr(args, "out", None):
        with open(args.out, "w") as f:
            json.dump(rep, f, indent=2)
    print(json.dumps(rep, indent=2))


def cmd_doctor(args, cfg):
    from ..probe import doctor
    rep = doctor()
    print(json.dumps(rep, indent=2))
    sys.exit(0 if all(c["ok"] for c in rep["checks"]) else 1)


def cmd_bundle(args, cfg):
    """Redacted diagnostic bundle (config with origins, versions, metrics, flight recorder,
    crash records, the doctor report)."""
    from ..daemon.bundle import make_bundle
    print(make_bundle(args.out, cfg, crash_dir=args.crash_dir, include_probe=args.probe))


def cmd_bench(args, cfg):
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.execv(sys.executable, [sys.executable, os.path.join(root, "bench.py")] + args.rest)


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if argv and argv[0] == "__runner":
        # hidden mode: the runner process a daemon's RunnerHost spawns (daemon/runner_proc.py)
        rp = argparse.ArgumentParser(prog="syntropy_b200 __runner")
        rp.add_argument("--ipc-fd", type=int, required=True)
        rp.add_argument("--region", required=True)
        ra = rp.parse_args(argv[1:])
        from ..daemon.runner_proc import serve
        raise SystemExit(serve(ra.ipc_fd, ra.region))
    ap = argparse.ArgumentParser(prog="syntropy_b200")
    ap.add_argument("--config", default=None, help="TOML config file")
    ap.add_argument("-o", "--set", action="append", default=[], help="section.key=value override")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("version")
    p = sub.add_parser("config")
    p.add_argument("action", nargs="?", choices=["show", "get", "set"], default="show")
    p.add_argument("key", nargs="?")
    p.add_argument("value", nargs="?")
    p.add_argument("--file", default=None, help="TOML file that `set` edits (default: --config)")
    p = sub.add_parser("plan")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--ctx", type=int, default=2048)
    p.add_argument("--expert-cache-frac", type=float, default=None)
    p.add_argument("--explain", action="store_true")
    p.add_argument("--probe", default=None, help="probe report (JSON) to price the plan with")
    p = sub.add_parser("run")
    p.add_argument("--prompt", default="Hello")
    p.add_argument("--tokens", default="")
    p.add_argument("--max-tokens", type=int, default=16)
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--seed", type=int, default=None)
    p.add_argument("--json", action="store_true", help="constrain the output to one JSON object")
    p.add_argument("--choices", default=None, help="constrain the output to one of these '|'-separated strings")
    p.add_argument("--device", default="cuda:0")
    p = sub.add_parser("chat", help="interactive chat (one user turn per input line)")
    p.add_argument("--system", default=None)
    p.add_argument("--max-tokens", type=int, default=256)
    p.add_argument("--temperature", type=float, default=0.7)
    p.add_argument("--seed", type=int, default=None)
    p.add_argument("--input", default=None, help="read the turns from this file instead of stdin")
    p.add_argument("--json", action="store_true", help="print each reply as a JSON line")
    p.add_argument("--device", default="cuda:0")
    sub.add_parser("ps", help="runner processes on this host (from their shared-memory status headers)")
    p = sub.add_parser("ls", help="models in the local store")
    p.add_argument("--store", default=os.path.expanduser("~/.cache/syntropy_b200/store"))
    p.add_argument("--verify", action="store_true", help="re-check every file's SHA-256")
    p = sub.add_parser("serve")
    p.add_argument("--device", default="cuda:0")
    p = sub.add_parser("probe")
    p.add_argument("--full", action="store_true")
    p.add_argument("--out", default=None, help="also write the report to this file")
    sub.add_parser("doctor")
    p = sub.add_parser("bundle")
    p.add_argument("--out", default="syntropy-bundle.tar.gz")
    p.add_argument("--crash-dir", default=os.path.expanduser("~/.cache/syntropy_b200/crashes"))
    p.add_argument("--probe", action="store_true", help="include the doctor report (touches the GPU)")
    p = sub.add_parser("bench")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    p = sub.add_parser("netprobe", help="network probe between two machines (listen | run | check)")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    args = ap.parse_args(argv)
    if args.cmd == "netprobe":
        from ..net.probe import main as netprobe_main
        raise SystemExit(netprobe_main(args.rest))
    from ..config import load_config
    cfg = load_config(args.config, overrides=args.set)
    {"version": cmd_version, "config": cmd_config, "plan": cmd_plan, "run": cmd_run, "chat": cmd_chat, "ls": cmd_ls, "ps": cmd_ps,
     "serve": cmd_serve,
     "probe": cmd_probe, "doctor": cmd_doctor, "bundle": cmd_bundle, "bench": cmd_bench}[args.cmd](args, cfg)


if __name__ == "__main__":
    main()
