"""KV tiering by preemption on CPU: with a page pool too small for every running sequence to
grow, the engine swaps the newest sequences' KV pages out to host memory and back in later;
the tokens equal a run with an ample pool."""
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def test_swap_out_and_in_keeps_tokens():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=2)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (20, 14, 30)]
    params = [SamplingParams(max_tokens=40), SamplingParams(max_tokens=40, temperature=0.7, seed=5),
              SamplingParams(max_tokens=40)]
    want = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(prompts, params)
    small = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, num_blocks=9))
    free0 = small.runner.kv.alloc.num_free
    got = small.generate(prompts, params)
    assert got == want
    assert small.stats["swapped_out"] > 0 and small.stats["swapped_in"] == small.stats["swapped_out"]
    assert small.runner.kv.alloc.num_free == free0  # every page returned
