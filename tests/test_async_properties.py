"""The serving loop under concurrency (CPU): requests submitted at once from asyncio tasks —
greedy, seeded sampling, penalised, constrained — each stream exactly the tokens the request
gets alone, while another request is cancelled mid-stream and its pages return to the pool."""
import asyncio

import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.async_engine import AsyncEngine
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def _mw():
    cfg = get_config("tiny-llama")
    return cfg, prepare_weights(cfg, torch.device("cpu"), seed=8)


def test_concurrent_streams_match_solo_runs():
    cfg, mw = _mw()
    g = torch.Generator().manual_seed(1)
    reqs = []
    for i in range(6):
        prompt = torch.randint(3, cfg.vocab, (int(torch.randint(3, 25, (1,), generator=g)),), generator=g).tolist()
        sp = [SamplingParams(max_tokens=12), SamplingParams(max_tokens=10, temperature=0.8, seed=i),
              SamplingParams(max_tokens=9, presence_penalty=1.0),
              SamplingParams(max_tokens=8, constraint={"choices": ["yes", "no"]})][i % 4]
        reqs.append((prompt, sp))
    solo = LLMEngine(ModelRunner(mw, max_batch=1, max_seq_len=64))
    want = [solo.generate([p], sp)[0] for p, sp in reqs]

    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=64, num_blocks=14), prefix_cache=True)
    free0 = eng.runner.kv.alloc.num_free
    aeng = AsyncEngine(eng)

    async def one(p, sp):
        toks = []
        async for ev in aeng.generate(p, sp):
            if ev.kind == "tokens":
                toks += ev.tokens
            if ev.kind == "error":
                raise RuntimeError(ev.error)
        return toks

    async def cancelled():
        n = 0
        async for ev in aeng.generate([4, 5, 6, 7], SamplingParams(max_tokens=40)):
            if ev.kind == "tokens":
                n += len(ev.tokens)
                if n >= 3:
                    return n  # leaving the stream cancels the request

    async def main():
        return await asyncio.gather(cancelled(), *[one(p, sp) for p, sp in reqs])

    try:
        res = asyncio.run(main())
    finally:
        aeng.close()
    assert res[0] >= 3
    assert res[1:] == want
    cached = eng.prefix.size if eng.prefix is not None else 0
    assert eng.runner.kv.alloc.num_free + cached == free0  # every page back (or held by the prefix cache)
