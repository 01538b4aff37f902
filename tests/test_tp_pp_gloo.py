"""Tensor x pipeline parallelism on CPU ranks (gloo, TP=2 x PP=2 over 4 ranks): each stage
holds half the layers, sharded over its two TP ranks; tokens equal a single process, for the
dense tiny Llama and for the tiny Qwen3-MoE (TP inside the experts)."""
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
    g = torch.Generator().manual_seed(21)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (9, 14, 3)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, model="tiny-llama"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from syntropy_b200.parallel.dist import init_distributed, shutdown, split_tp_pp
    from syntropy_b200.parallel.pp import PPGroup
    from syntropy_b200.parallel.tp import TPGroup
    ctx = init_distributed(backend="gloo", timeout_s=60)
    cfg = get_config(model).replace(n_layers=4)
    sd = synthetic_state_dict(cfg, seed=13)
    tp_ctx, pp_group, pp_ranks, stage = split_tp_pp(ctx, 2, 2)
    pp = PPGroup(ctx, 2, stage, cfg.n_layers, group=pp_group, ranks=pp_ranks)
    mw = prepare_weights(cfg, "cpu", state_dict=sd, tp=(tp_ctx.rank, 2), layer_range=pp.layer_range)
    tp = TPGroup(tp_ctx, cfg.hidden, cap=4, n_layers=len(mw.layers), fused=False)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, tp=tp, pp=pp))
    outs = eng.generate(_prompts(), SamplingParams(max_tokens=5, temperature=0.7, seed=9))
    q.put((rank, outs))
    shutdown(ctx)


def test_tp2_pp2_match_single_process(model="tiny-llama"):
    cfg = get_config(model).replace(n_layers=4)
    sd = synthetic_state_dict(cfg, seed=13)
    want = LLMEngine(ModelRunner(prepare_weights(cfg, "cpu", state_dict=sd), max_batch=4, max_seq_len=128)).generate(
        _prompts(), SamplingParams(max_tokens=5, temperature=0.7, seed=9))
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, model)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got[0] == got[1] == got[2] == got[3] == want


def test_tp2_pp2_moe_match_single_process():
    """The same with the tiny Qwen3-MoE: experts split along their width inside each stage."""
    test_tp2_pp2_match_single_process("tiny-qwen-moe")
