"""Host CPU expert tier on a B200: with half of the VRAM-capped host experts computed by CPU
threads (mailbox hand-off captured in the decode graphs), greedy tokens equal the all-GPU
path's; the CPU really served pairs; and a hand-off nobody answers ends in a status error
after the time limit instead of a hang."""
import pytest
import torch

from syntropy_b200.core.errors import SynError
from syntropy_b200.experts.cache import ExpertCache
from syntropy_b200.experts.cpu_tier import CpuExpertTier
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

pytestmark = pytest.mark.gpu


def _engine(cuda, share, graphs=True, timeout_s=2.0):
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=21)
    cache = ExpertCache(mw.layers, 0.5, cuda)
    runner = ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=graphs)
    runner.expert_cache = cache
    # mode 1 (BF16, exact products): the tokens must equal the GPU-only engine
    tier = CpuExpertTier(cache, cfg, max_rows=runner.max_batch, cpu_share=share, threads=4,
                         timeout_s=timeout_s, mode=1) if share else None
    return LLMEngine(runner), cfg, tier


def _prompts(cfg):
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (17, 40, 5, 64)]


def test_cpu_tier_matches_gpu_path(cuda):
    eng, cfg, _ = _engine(cuda, 0.0)
    want = eng.generate(_prompts(cfg), SamplingParams(max_tokens=8))
    eng, cfg, tier = _engine(cuda, 0.5)
    try:
        got = eng.generate(_prompts(cfg), SamplingParams(max_tokens=8))
        st = tier.stats()
    finally:
        tier.close()
    assert got == want
    assert st["jobs"] > 0 and st["pairs"] > 0
    b = tier.cache.banks[0]
    assert b.cpu_owned and all(b.slot_of[e] < 0 for e in b.cpu_owned)
    assert all(int(b.gu.qw_ptrs[e]) == 0 for e in b.cpu_owned)


def test_unanswered_handoff_times_out(cuda):
    eng, cfg, tier = _engine(cuda, 0.5, graphs=False, timeout_s=0.2)
    tier.close()  # nobody answers the mailbox now
    eng.add_request(_prompts(cfg)[0], SamplingParams(max_tokens=4))
    eng.step()  # prefill (GPU only)
    with pytest.raises(SynError, match="no answer"):
        eng.step()  # decode: every MoE layer's wait runs out after 0.2 s
    torch.cuda.synchronize()  # the context is still usable
    assert int(tier.status.item()) == 0
