"""Logit processing on CPU (penalties and bias, re-drawn after the step with the same draw
counter): a large bias forces its token, a large frequency penalty forbids repeats, a large
repetition penalty steers greedy decoding away from every token already seen, and the default
parameters leave the output unchanged."""
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def _engine():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=0)
    return LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=256)), cfg


def test_penalties_and_bias():
    eng, cfg = _engine()
    prompt = [5, 9, 17, 33, 5, 9]
    base = eng.generate([prompt], SamplingParams(max_tokens=24))[0]
    assert eng.generate([prompt], SamplingParams(max_tokens=24, logit_bias={}))[0] == base
    forced = eng.generate([prompt], SamplingParams(max_tokens=6, logit_bias={77: 1e4}))[0]
    assert forced == [77] * 6
    nodup = eng.generate([prompt], SamplingParams(max_tokens=24, frequency_penalty=1e4))[0]
    assert len(set(nodup)) == len(nodup)
    fresh = eng.generate([prompt], SamplingParams(max_tokens=16, repetition_penalty=1e6))[0]
    seen = set(prompt)
    for t in fresh:
        assert t not in seen
        seen.add(t)
    # sampled rows: the processed draw is reproducible under a client seed
    a = eng.generate([prompt], SamplingParams(max_tokens=12, temperature=0.9, seed=7, presence_penalty=2.0))[0]
    b = eng.generate([prompt], SamplingParams(max_tokens=12, temperature=0.9, seed=7, presence_penalty=2.0))[0]
    assert a == b
