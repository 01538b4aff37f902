"""Speculative decoding with a draft model on CPU: greedy output equals plain decoding (exact
acceptance), a draft model identical to the target has every draft accepted, a different
draft model still gives the target's tokens, and finished sequences return their draft pages."""
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner
from syntropy_b200.runtime.spec import DraftModelDrafter, SpecConfig


def _prompts(vocab):
    g = torch.Generator().manual_seed(4)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in (10, 23, 5)]


def test_draft_model_spec_matches_plain():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=3)
    params = SamplingParams(max_tokens=20)
    want = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128)).generate(_prompts(cfg.vocab), params)

    same = DraftModelDrafter(ModelRunner(mw, max_batch=8, max_seq_len=160))
    eng = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128), spec=SpecConfig(gamma=3, drafter=same))
    assert eng.generate(_prompts(cfg.vocab), params) == want
    assert eng.acceptance_rate > 0.95
    free = same.r.kv.alloc.num_free
    assert not same.blocks and free == ModelRunner(mw, max_batch=8, max_seq_len=160).kv.alloc.num_free

    other = DraftModelDrafter(ModelRunner(prepare_weights(cfg, torch.device("cpu"), seed=11), max_batch=8,
                                          max_seq_len=160))
    eng2 = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128), spec=SpecConfig(gamma=2, drafter=other))
    assert eng2.generate(_prompts(cfg.vocab), params) == want
