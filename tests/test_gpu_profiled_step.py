"""Profiled decode steps: the timestamped graph variant gives the same tokens as the plain
one and reports a positive device time for every layer segment."""
import pytest
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

pytestmark = pytest.mark.gpu


def test_profiled_step(cuda):
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=4)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (9, 30)]
    sp = SamplingParams(max_tokens=6)
    want = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(prompts, sp)
    runner = ModelRunner(mw, max_batch=4, max_seq_len=128)
    eng = LLMEngine(runner)
    ids = [eng.add_request(p, sp) for p in prompts]
    eng.step()  # prefill
    runner.profile_next = True
    eng.step()  # profiled decode step
    prof = runner.step_profile()
    while eng.has_work():
        eng.step()
    assert [eng.finished[i].output for i in ids] == want
    labels = [lab for lab, _ in prof]
    assert labels[0] == "layer0.attention" and labels[-1] == "sample"
    # per MoE layer: attention, route, gate_up, down, moe (combine); then lm_head and sample
    assert len(labels) == 5 * cfg.n_layers + 2
    assert [lab.split(".")[-1] for lab in labels[:5]] == ["attention", "route", "gate_up", "down", "moe"]
    assert all(ms > 0 for _, ms in prof)
