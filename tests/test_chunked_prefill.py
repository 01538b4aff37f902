"""Chunked prefill with decode-first steps (reference plan/rfcs/RFC-0012-execution-scheduler.md
:299-314): a long prompt enters the KV cache in chunks while the running sequences keep
decoding one token per step, and every request still gets exactly the tokens it gets alone."""
import random

import pytest
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


@pytest.fixture(scope="module")
def model():
    cfg = get_config("tiny-llama")
    return cfg, prepare_weights(cfg, "cpu", seed=0, max_pos=512)


def _engine(model, chunk=None, prefix=False, max_batch=4):
    cfg, mw = model
    return LLMEngine(ModelRunner(mw, max_batch=max_batch, max_seq_len=480), chunk_tokens=chunk, prefix_cache=prefix)


def _alone(model, prompt, params):
    return _engine(model).generate([prompt], params)[0]


def test_long_prompt_stalls_running_sequences_by_one_chunk_at_most(model):
    cfg, _ = model
    g = torch.Generator().manual_seed(1)
    short = torch.randint(0, cfg.vocab, (12,), generator=g).tolist()
    long = torch.randint(0, cfg.vocab, (300,), generator=g).tolist()
    sp = SamplingParams(max_tokens=40, temperature=0.0)
    eng = _engine(model, chunk=32)
    eng.step_log = []
    a = eng.add_request(short, sp)
    eng.step()  # the short prompt is prefilled and running
    b = eng.add_request(long, SamplingParams(max_tokens=6, temperature=0.0))
    emitted = []
    while eng.has_work():
        before = len(eng.running and [s for s in eng.running if s.seq_id == a] and
                     [s for s in eng.running if s.seq_id == a][0].output or [])
        eng.step()
        s_a = eng.finished.get(a) or next(s for s in eng.running if s.seq_id == a)
        emitted.append(len(s_a.output) - before)
        if a in eng.finished:
            break
    # while the long prompt was being prefilled (10 chunks of 32), the running sequence got a
    # token on every step, and no step prefilled more than one chunk
    assert all(n == 1 for n in emitted)
    assert max(p for _, p in eng.step_log) <= 32
    assert sum(1 for d, p in eng.step_log if d and p) >= 9  # mixed steps: decode rows + a chunk
    while eng.has_work():
        eng.step()
    assert eng.finished[a].output == _alone(model, short, sp)
    assert eng.finished[b].output == _alone(model, long, SamplingParams(max_tokens=6, temperature=0.0))


@pytest.mark.parametrize("seed", range(4))
def test_random_mixes_equal_solo_runs(model, seed):
    """Random arrivals of prompts of random lengths (some sharing prefixes through the prefix
    cache), sampled and greedy, chunk sizes from 1 to 64: each request's tokens equal its solo
    run's (the sampling key is per request, so batch-mates never change a draw)."""
    cfg, _ = model
    rng = random.Random(seed)
    chunk = rng.choice([1, 7, 16, 64])
    base = [rng.randrange(cfg.vocab) for _ in range(40)]
    reqs = []
    for i in range(6):
        n = rng.randrange(3, 120)
        p = (base[:rng.randrange(16, 40)] if rng.random() < 0.5 else []) + [rng.randrange(cfg.vocab) for _ in range(n)]
        sp = SamplingParams(max_tokens=rng.randrange(1, 12), temperature=rng.choice([0.0, 0.8]), seed=1000 + i)
        reqs.append((rng.randrange(0, 20), p, sp))
    eng = _engine(model, chunk=chunk, prefix=True)
    ids, t = {}, 0
    pending = sorted(range(len(reqs)), key=lambda i: reqs[i][0])
    while pending or eng.has_work():
        while pending and reqs[pending[0]][0] <= t:
            i = pending.pop(0)
            ids[i] = eng.add_request(reqs[i][1], reqs[i][2])
        eng.step()
        t += 1
    for i, (_, p, sp) in enumerate(reqs):
        assert eng.finished[ids[i]].output == _alone(model, p, sp), (i, chunk)


def test_abort_while_prefilling_returns_pages(model):
    cfg, _ = model
    eng = _engine(model, chunk=8)
    free0 = eng.runner.kv.alloc.num_free
    sid = eng.add_request(list(range(100)), SamplingParams(max_tokens=4))
    eng.step()
    assert eng.prefilling and eng.prefilling[0].prefilled == 8
    eng.abort(sid)
    assert not eng.prefilling and eng.finished[sid].finish_reason == "cancelled"
    assert eng.runner.kv.alloc.num_free == free0
