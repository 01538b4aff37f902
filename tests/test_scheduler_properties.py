"""Scheduling properties (hypothesis, CPU): for random mixes of requests on a tight KV page
pool — with or without the prefix cache and n-gram speculation — every request finishes within
a bounded number of steps and greedy outputs equal those of the same request served alone with
an ample pool (preemption, prefix sharing and batching never change tokens).  Sampled requests
(client seed), penalised ones and choice-constrained ones keep that property: draws are keyed
by (seed, stream, counter), never by batch position."""
import pytest
import torch

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from syntropy_b200.models.config import get_config  # noqa: E402
from syntropy_b200.models.transformer import prepare_weights  # noqa: E402
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams  # noqa: E402
from syntropy_b200.runtime.runner import ModelRunner  # noqa: E402
from syntropy_b200.runtime.spec import SpecConfig  # noqa: E402

_MW = {}


def _mw():
    if "mw" not in _MW:
        cfg = get_config("tiny-llama")
        _MW["cfg"], _MW["mw"] = cfg, prepare_weights(cfg, torch.device("cpu"), seed=6)
        # reference: each request alone with an ample pool (speculation on or off, like the run:
        # with sampling, speculative decoding is exact in distribution but takes other draws)
        _MW[False] = LLMEngine(ModelRunner(_MW["mw"], max_batch=1, max_seq_len=96))
        _MW[True] = LLMEngine(ModelRunner(_MW["mw"], max_batch=3, max_seq_len=96), spec=SpecConfig(gamma=2))
    return _MW["cfg"], _MW["mw"]


def _params(kind, m, seed):
    if kind == 1:
        return SamplingParams(max_tokens=m, temperature=0.9, top_p=0.95, seed=seed)
    if kind == 2:
        return SamplingParams(max_tokens=m, frequency_penalty=1.5, logit_bias={7: 2.0})
    if kind == 3:
        return SamplingParams(max_tokens=m, temperature=0.7, seed=seed, constraint={"choices": ["ab", "abc", "x"]})
    return SamplingParams(max_tokens=m)


def _alone(prompt, params, spec):
    _mw()
    return _MW[spec].generate([prompt], params)[0]


@settings(max_examples=25, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(reqs=st.lists(st.tuples(st.integers(0, 2), st.integers(1, 30), st.integers(1, 24), st.integers(0, 3),
                               st.integers(0, 99)), min_size=1, max_size=5),
       pool=st.integers(7, 14), prefix=st.booleans(), spec=st.booleans())
def test_every_request_finishes_with_its_own_tokens(reqs, pool, prefix, spec):
    cfg, mw = _mw()
    bases = [[11, 12, 13, 14, 15, 16, 17, 18, 19, 20, 21, 22, 23, 24, 25, 26, 27], [40, 41], [90]]
    prompts = [bases[b] + list(range(100, 100 + n)) for b, n, *_ in reqs]
    params = [_params(kind, m, seed) for _, _, m, kind, seed in reqs]
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=96, num_blocks=pool), prefix_cache=prefix,
                    spec=SpecConfig(gamma=2) if spec else None)
    ids = []
    for p, sp in zip(prompts, params):
        try:
            ids.append(eng.add_request(p, sp))
        except ValueError:  # larger than the whole pool: rejected up front
            ids.append(None)
    for _ in range(400):
        if not eng.has_work():
            break
        eng.step()
    assert not eng.has_work(), (len(eng.running), len(eng.waiting), len(eng.swapped))
    for i, p, sp in zip(ids, prompts, params):
        if i is not None:
            assert eng.finished[i].output == _alone(p, sp, spec)


@settings(max_examples=15, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(n=st.integers(1, 30), m=st.integers(2, 20), cut=st.integers(0, 19), kind=st.integers(0, 3),
       seed=st.integers(0, 99))
def test_saved_session_resumes_exactly(n, m, cut, kind, seed):
    """A sequence saved at any step and restored into a fresh engine (with other traffic there)
    finishes with the tokens of an uninterrupted run (a constrained one with its grammar state)."""
    cfg, mw = _mw()
    prompt = [5, 6, 7] + list(range(200, 200 + n))
    sp = _params(kind, m, seed)
    want = _alone(prompt, sp, False)
    a = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=96))
    sid = a.add_request(prompt, sp)
    a.step()  # prefill: first token
    for _ in range(min(cut, m - 2)):
        a.step()
    if sid in a.finished:
        assert a.finished[sid].output == want
        return
    state = a.save_session(sid)
    b = LLMEngine(ModelRunner(mw, max_batch=3, max_seq_len=96))
    other = b.add_request([9, 9, 9, 9], SamplingParams(max_tokens=5))
    rid = b.restore_session(state)
    while b.has_work():
        b.step()
    assert b.finished[rid].output == want
    assert len(b.finished[other].output) == 5
