"""Hot-path guard on a B200: once the decode graphs are captured, decode steps through the
engine make no device allocation (the caching allocator's request count does not move) —
the step is a descriptor upload and a graph replay."""
import pytest
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

pytestmark = pytest.mark.gpu


def test_decode_steps_allocate_nothing(cuda):
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=1)
    eng = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=True))
    g = torch.Generator().manual_seed(2)
    for n in (11, 30, 7, 19):
        eng.add_request(torch.randint(0, cfg.vocab, (n,), generator=g).tolist(), SamplingParams(max_tokens=40))
    for _ in range(6):  # prefill, then decode steps that capture the graph of this bucket
        eng.step()
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats()["allocation.all.allocated"]
    steps = 0
    while len(eng.running) == 4 and steps < 20:
        eng.step()
        steps += 1
    torch.cuda.synchronize()
    after = torch.cuda.memory_stats()["allocation.all.allocated"]
    assert steps == 20
    assert after == before, f"{after - before} device allocations in {steps} decode steps"
