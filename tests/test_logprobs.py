"""Per-token logprobs: the emitted token's log-probability and the top alternatives equal the
f32 reference forward's log-softmax at each position; asking for them changes no token."""
import pytest
import torch

from syntropy_b200.models import reference
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_logprobs_match_reference(temperature):
    cfg = get_config("tiny-llama")
    sd = synthetic_state_dict(cfg, seed=0)
    mw = prepare_weights(cfg, "cpu", state_dict=sd, max_pos=96)
    prompts = [[5, 17, 99, 3], [7, 8]]
    base = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=64)).generate(
        prompts, SamplingParams(max_tokens=6, temperature=temperature, seed=3))
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=64))
    ids = [eng.add_request(p, SamplingParams(max_tokens=6, temperature=temperature, seed=3,
                                             logprobs=3 if i == 0 else None)) for i, p in enumerate(prompts)]
    while eng.has_work():
        eng.step()
    s0 = eng.finished[ids[0]]
    assert eng.finished[ids[1]].logprobs == []  # rows that did not ask record nothing
    assert s0.output == base[0]  # asking for logprobs changes nothing
    assert len(s0.logprobs) == len(s0.output)
    full = torch.tensor(prompts[0] + s0.output)
    ref = torch.log_softmax(reference.forward(full, sd, cfg).float(), -1)
    for j, rec in enumerate(s0.logprobs):
        row = ref[len(prompts[0]) - 1 + j]
        assert rec["token"] == s0.output[j]
        assert abs(rec["logprob"] - row[rec["token"]].item()) < 1e-3
        top = row.topk(3)
        assert [t for t, _ in rec["top"]] == top.indices.tolist()
        assert all(abs(v - w) < 1e-3 for (_, v), w in zip(rec["top"], top.values.tolist()))
        if temperature == 0.0:
            assert rec["top"][0][0] == rec["token"]


def test_logprobs_rejected_with_speculation():
    from syntropy_b200.runtime.spec import NgramDrafter, SpecConfig
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, "cpu", max_pos=64)
    eng = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=48), spec=SpecConfig(gamma=2, drafter=NgramDrafter()))
    with pytest.raises(ValueError, match="logprobs"):
        eng.add_request([1, 2, 3], SamplingParams(max_tokens=4, logprobs=1))


def test_logprobs_count_is_capped():
    """Counts outside 0..20 (or above the vocabulary) are refused at intake; the cap itself works."""
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, "cpu", max_pos=64)
    eng = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=48))
    for bad in (-1, 21, 10 ** 6, True, 1.5):
        with pytest.raises(ValueError, match="logprobs"):
            eng.add_request([1, 2, 3], SamplingParams(max_tokens=2, logprobs=bad))
    sid = eng.add_request([1, 2, 3], SamplingParams(max_tokens=2, logprobs=20))
    while eng.has_work():
        eng.step()
    assert all(len(r["top"]) == 20 for r in eng.finished[sid].logprobs)


def test_logprobs_rejected_under_pipeline_parallelism():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, "cpu", max_pos=64)
    runner = ModelRunner(mw, max_batch=2, max_seq_len=48)
    runner.pp = object()  # any pipeline group: the intake check only looks for its presence
    eng = LLMEngine(runner)
    with pytest.raises(ValueError, match="pipeline"):
        eng.add_request([1, 2, 3], SamplingParams(max_tokens=2, logprobs=1))
