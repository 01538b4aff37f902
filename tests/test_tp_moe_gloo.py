"""Tensor parallelism inside the experts on CPU ranks (gloo, world size 2): every expert and the
router-replicated MoE layers of the tiny Qwen3-MoE split along the expert FFN width, partial
outputs summed over the group, give the same greedy tokens as one process."""
import os
import socket

import torch
import torch.multiprocessing as mp

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def _prompts():
    g = torch.Generator().manual_seed(6)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (9, 2, 17)]


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
    from syntropy_b200.parallel.tp import TPGroup
    ctx = init_distributed(backend="gloo", timeout_s=60)
    cfg = get_config("tiny-qwen-moe")
    sd = synthetic_state_dict(cfg, seed=8)
    mw = prepare_weights(cfg, "cpu", state_dict=sd, tp=(rank, world))
    tp = TPGroup(ctx, cfg.hidden, cap=4, n_layers=cfg.n_layers, fused=False)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, tp=tp))
    outs = eng.generate(_prompts(), SamplingParams(max_tokens=6))
    q.put((rank, outs))
    shutdown(ctx)


def test_tp_experts_gloo_matches_single_process():
    cfg = get_config("tiny-qwen-moe")
    sd = synthetic_state_dict(cfg, seed=8)
    want = LLMEngine(ModelRunner(prepare_weights(cfg, "cpu", state_dict=sd), max_batch=4, max_seq_len=128)).generate(
        _prompts(), SamplingParams(max_tokens=6))
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got[0] == got[1] == want
