"""Speculative decoding: greedy verify windows give exactly the non-speculative greedy
tokens; the host acceptance oracle preserves the target distribution (chi-square style
check on a small vocabulary); n-gram drafter proposals."""
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner
from syntropy_b200.runtime.sampling_ref import verify_ref
from syntropy_b200.runtime.spec import NgramDrafter, SpecConfig


def test_ngram_drafter():
    d = NgramDrafter(3)
    assert d.propose([1, 2, 3, 4, 1, 2, 3], 2) == [4, 1]
    assert d.propose([5, 6, 7], 2) == [7, 7]


def test_greedy_spec_equals_plain():
    cfg = get_config("tiny-qwen-moe")
    mw = prepare_weights(cfg, "cpu", seed=3)
    g = torch.Generator().manual_seed(1)
    base = torch.randint(0, cfg.vocab, (8,), generator=g).tolist()
    prompts = [base * 3, torch.randint(0, cfg.vocab, (20,), generator=g).tolist()]
    want = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128)).generate(prompts, SamplingParams(max_tokens=12))
    eng = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128), spec=SpecConfig(gamma=3))
    got = eng.generate(prompts, SamplingParams(max_tokens=12))
    assert got == want
    assert eng.stats["spec_drafted"] > 0


def test_acceptance_preserves_distribution():
    torch.manual_seed(0)
    V, g, S = 6, 1, 4000
    target = torch.randn(V) * 1.5
    logits = target.repeat(S * (g + 1), 1)
    drafts = torch.full((S, g), 2, dtype=torch.int32)  # always draft token 2 (point mass)
    temp = torch.ones(S)
    topk = torch.zeros(S, dtype=torch.int32)
    topp = torch.ones(S)
    seed = torch.full((S,), 11, dtype=torch.int64)
    stream = torch.arange(S, dtype=torch.int64)
    ctr = torch.zeros(S, dtype=torch.int64)
    toks, nacc = verify_ref(logits, drafts, temp, topk, topp, seed, stream, ctr)
    first = toks[:, 0]
    freq = torch.bincount(first.long(), minlength=V).double() / S
    p = torch.softmax(target, 0).double()
    assert (freq - p).abs().max() < 0.03, (freq, p)
    # draws: accept -> 1 (u) + 1 (bonus); reject -> 1 (u) + 1 (residual)
    assert torch.all(ctr == 2)


def test_ngram_native_batch_matches_python_rule():
    """The native batched prompt-lookup drafts equal the per-sequence Python rule."""
    import random as _r
    from syntropy_b200.runtime.spec import NgramDrafter
    rng = _r.Random(7)
    d = NgramDrafter(n=3)
    hist = [[rng.randrange(6) for _ in range(rng.randrange(1, 60))] for _ in range(50)]
    hist.append([5])
    for g in (1, 3, 4):
        assert d.propose_batch(hist, g) == [d.propose(h, g) for h in hist]


def test_graph_bucket_never_exceeds_runner_rows():
    """A decode bucket holds the rows but never more than the runner's rows (the descriptor and
    the per-row buffers are sized by them), and the last bucket is the runner's own row count."""
    from syntropy_b200.runtime.runner import BUCKETS, bucket_for
    for cap in (1, 4, 50, 64, 100, 256):
        for n in range(1, cap + 1):
            b = bucket_for(n, cap=cap)
            assert n <= b <= cap
            assert b in BUCKETS or b == cap
    assert bucket_for(40) == 48 and bucket_for(200) == 256


class _WrongDrafter:
    """Drafts that are never the model's greedy token (vocab-1 - last token)."""

    def propose(self, history, g):
        return [(1023 - history[-1]) % 1024] * g


def test_low_acceptance_pauses_drafting_and_keeps_tokens():
    """With drafts that are always rejected the engine stops paying for verify windows: after
    `window` drafted tokens at low acceptance it takes `pause_steps` plain steps, then probes
    again; the greedy tokens equal plain decoding throughout."""
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=0)
    prompts = [[1, 2, 3, 4, 5, 6, 7, 8], [9, 10, 11]]
    params = SamplingParams(max_tokens=60)
    want = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128)).generate(prompts, params)
    spec = SpecConfig(gamma=3, drafter=_WrongDrafter(), window=24, pause_steps=5)
    eng = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128), spec=spec)
    assert eng.generate(prompts, params) == want
    assert eng.stats["spec_paused_steps"] >= 5
    assert eng.stats["spec_accepted"] <= 0.1 * eng.stats["spec_drafted"] + 6
    # min_accept 0 turns the pause off: every step drafts
    eng2 = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=128),
                     spec=SpecConfig(gamma=3, drafter=_WrongDrafter(), min_accept=0.0))
    assert eng2.generate(prompts, params) == want and eng2.stats["spec_paused_steps"] == 0
