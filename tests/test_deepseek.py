"""DeepSeek-V3 family on CPU: MLA (absorbed, paged latent cache), group-limited sigmoid
routing with a shared expert and dense leading layers; greedy tokens equal the naive f32
reference forward; MTP drafting with exact verification equals plain greedy decoding."""
import torch

from syntropy_b200.models import reference
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def test_deepseek_greedy_matches_reference():
    cfg = get_config("tiny-deepseek")
    sd = synthetic_state_dict(cfg, seed=5)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg.vocab, (21,), generator=g).tolist()
    want = reference.greedy_generate(torch.tensor(prompt), sd, cfg, 8)
    mw = prepare_weights(cfg, "cpu", state_dict=sd)
    got = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate([prompt], SamplingParams(max_tokens=8))
    assert got[0] == want


def test_mtp_spec_greedy_equals_plain_and_reports_acceptance():
    from syntropy_b200.runtime.spec import MTPDrafter, SpecConfig
    cfg = get_config("tiny-deepseek")
    mw = prepare_weights(cfg, "cpu", seed=6)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (13, 30)]
    want = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128)).generate(prompts, SamplingParams(max_tokens=10))
    runner = ModelRunner(mw, max_batch=8, max_seq_len=128)
    eng = LLMEngine(runner, spec=SpecConfig(drafter=MTPDrafter(runner)))
    got = eng.generate(prompts, SamplingParams(max_tokens=10))
    assert got == want
    assert eng.stats["spec_drafted"] > 0 and 0.0 <= eng.acceptance_rate <= 1.0
