"""Expert parallelism on CPU ranks (gloo, world size 2): the NCCL-baseline data plane
(all-gather rows, local experts, reduce-scatter) with lockstep engine steps gives the same
greedy tokens as one process holding every expert."""
import os
import socket

import torch
import torch.multiprocessing as mp

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

CFG = "tiny-qwen-moe"


def _prompts():
    g = torch.Generator().manual_seed(7)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (9, 21, 5, 14)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from syntropy_b200.parallel.dist import init_distributed, shutdown
    from syntropy_b200.parallel.ep import EPGroup
    ctx = init_distributed(backend="gloo", timeout_s=60)
    cfg = get_config(CFG)
    sd = synthetic_state_dict(cfg, seed=11)
    ep = EPGroup(ctx, cfg.n_experts, cfg.top_k, cfg.hidden, cap=8, n_layers=cfg.n_layers, fused=False)
    mw = prepare_weights(cfg, "cpu", state_dict=sd, expert_range=ep.expert_range)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, ep=ep), dist_ctx=ctx)
    mine = _prompts()[rank::world]
    outs = eng.generate(mine, SamplingParams(max_tokens=6))
    q.put((rank, outs))
    shutdown(ctx)


def test_ep_baseline_gloo_matches_single_process():
    cfg = get_config(CFG)
    sd = synthetic_state_dict(cfg, seed=11)
    mw = prepare_weights(cfg, "cpu", state_dict=sd)
    want = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(_prompts(), SamplingParams(max_tokens=6))
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, outs = q.get(timeout=300)
        got[r] = outs
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert got[r] == want[r::world], (r, got[r], want[r::world])
