"""Qwen2-style dense variant on CPU: bias on the Q, K and V projections and tied embeddings.
The engine's greedy tokens equal the naive f32 reference forward; tensor parallelism (gloo,
2 ranks) slices the biases with their heads and gives the same tokens."""
import os
import socket

import torch
import torch.multiprocessing as mp

from syntropy_b200.models import reference
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def _prompt():
    return torch.randint(0, 1024, (13,), generator=torch.Generator().manual_seed(7)).tolist()


def test_qkv_bias_matches_reference():
    cfg = get_config("tiny-qwen2")
    sd = synthetic_state_dict(cfg, seed=5)
    assert "layers.0.q_bias" in sd and "lm_head" not in sd
    want = reference.greedy_generate(torch.tensor(_prompt()), sd, cfg, 12)
    eng = LLMEngine(ModelRunner(prepare_weights(cfg, "cpu", state_dict=sd), max_batch=2, max_seq_len=64))
    got = eng.generate([_prompt()], SamplingParams(max_tokens=12))[0]
    assert got == list(want)
    # parameter count (norm scales aside) includes the projection biases
    assert cfg.param_count() == sum(t.numel() for n, t in sd.items() if not n.endswith("norm"))


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
    cfg = get_config("tiny-qwen2")
    mw = prepare_weights(cfg, "cpu", state_dict=synthetic_state_dict(cfg, seed=5), tp=(rank, world))
    tp = TPGroup(ctx, cfg.hidden, cap=2, n_layers=cfg.n_layers, fused=False)
    out = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=64, tp=tp)).generate([_prompt()],
                                                                                  SamplingParams(max_tokens=12))
    q.put((rank, out[0]))
    shutdown(ctx)


def test_qkv_bias_under_tensor_parallelism():
    cfg = get_config("tiny-qwen2")
    sd = synthetic_state_dict(cfg, seed=5)
    want = list(reference.greedy_generate(torch.tensor(_prompt()), sd, cfg, 12))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[0] == got[1] == want
