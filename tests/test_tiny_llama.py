"""Plumbing gate on CPU: the tiny Llama-style decoder (2 layers, hidden 256, GQA 4/2,
head_dim 64, SwiGLU 688, vocab 1024, f32 N(0, 0.02) weights, seed 0), batch 1, a
32-token uniform prompt, greedy decode of 32 tokens through the paged-KV engine equals the
naive f32 reference forward."""
import torch

from syntropy_b200.models import reference
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def _prompt(n, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def test_tiny_llama_greedy_matches_reference():
    cfg = get_config("tiny-llama")
    sd = synthetic_state_dict(cfg, seed=0)
    prompt = _prompt(32, cfg.vocab)
    want = reference.greedy_generate(torch.tensor(prompt), sd, cfg, 32)
    mw = prepare_weights(cfg, "cpu", state_dict=sd)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128))
    got = eng.generate([prompt], SamplingParams(max_tokens=32))[0]
    assert got == want


def test_tiny_qwen_moe_greedy_matches_reference():
    cfg = get_config("tiny-qwen-moe")
    sd = synthetic_state_dict(cfg, seed=1)
    prompt = _prompt(16, cfg.vocab, 1)
    want = reference.greedy_generate(torch.tensor(prompt), sd, cfg, 12)
    mw = prepare_weights(cfg, "cpu", state_dict=sd)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128))
    got = eng.generate([prompt], SamplingParams(max_tokens=12))[0]
    assert got == want


def test_batched_decode_equals_single():
    cfg = get_config("tiny-qwen-moe")
    sd = synthetic_state_dict(cfg, seed=2)
    prompts = [_prompt(n, cfg.vocab, n) for n in (5, 17, 33)]
    mw = prepare_weights(cfg, "cpu", state_dict=sd)
    single = [LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate([p], SamplingParams(max_tokens=8))[0]
              for p in prompts]
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128))
    batched = eng.generate(prompts, SamplingParams(max_tokens=8))
    assert batched == single
