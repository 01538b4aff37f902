"""Speculative decoding with stochastic drafts (reference plan/rfcs/RFC-0012-execution-
scheduler.md:612-613): a draft d ~ q is accepted with probability min(1, p(d) / q(d)); on
rejection the token is drawn from norm(max(0, p - q)).  The emitted tokens then follow the
target distribution p exactly, whatever q is.  Checked with chi-square tests: on the acceptance
rule itself (toy distributions, many windows), and end to end (a draft model sampling at its
own temperature against plain sampling of the target, RFC-0012:804)."""
import math

import numpy as np
import pytest
import torch

scipy_stats = pytest.importorskip("scipy.stats")

from syntropy_b200.models.config import get_config  # noqa: E402
from syntropy_b200.models.transformer import prepare_weights  # noqa: E402
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams  # noqa: E402
from syntropy_b200.runtime.runner import ModelRunner  # noqa: E402
from syntropy_b200.runtime.sampling_ref import verify_ref  # noqa: E402
from syntropy_b200.runtime.spec import DraftModelDrafter, SpecConfig  # noqa: E402


def _chi2_fit(counts, probs):
    counts = np.asarray(counts, dtype=np.float64)
    exp = np.asarray(probs, dtype=np.float64) * counts.sum()
    keep = exp > 0
    return scipy_stats.chisquare(counts[keep], exp[keep] * counts[keep].sum() / exp[keep].sum()).pvalue


def test_stochastic_rule_preserves_the_target_distribution():
    V, g, n = 6, 2, 6000
    p_logits = torch.tensor([[2.0, 1.0, 0.5, 0.0, -1.0, 0.3],
                             [0.0, 1.5, 1.5, -0.5, 0.2, 0.1],
                             [1.0, 0.0, 0.0, 0.0, 0.0, 2.0]])
    q = torch.tensor([[0.05, 0.40, 0.05, 0.30, 0.10, 0.10],
                      [0.30, 0.10, 0.20, 0.20, 0.10, 0.10]])
    p = torch.softmax(p_logits, -1)
    rng = np.random.default_rng(0)
    first = np.zeros(V)
    second = np.zeros(V)
    acc0 = 0
    for t in range(n):
        d = torch.tensor([[int(rng.choice(V, p=q[j].numpy())) for j in range(g)]], dtype=torch.int32)
        ctr = torch.tensor([t * 16], dtype=torch.int64)
        toks, nacc = verify_ref(p_logits, d, torch.tensor([1.0]), torch.tensor([0], dtype=torch.int32),
                                torch.tensor([1.0]), torch.tensor([7], dtype=torch.int64),
                                torch.tensor([3], dtype=torch.int64), ctr, draft_probs=q[None])
        first[int(toks[0, 0])] += 1
        if int(nacc[0]) >= 1:
            acc0 += 1
            second[int(toks[0, 1])] += 1
    assert _chi2_fit(first, p[0]) > 1e-3
    assert _chi2_fit(second, p[1]) > 1e-3
    # acceptance at the first position: sum_v min(p, q)
    a = float(torch.minimum(p[0], q[0]).sum())
    assert abs(acc0 / n - a) < 4 * math.sqrt(a * (1 - a) / n)


def test_draft_equal_to_target_is_always_accepted():
    V = 5
    p_logits = torch.randn(3, V)
    q = torch.softmax(p_logits[:2], -1)
    d = torch.tensor([[1, 3]], dtype=torch.int32)
    toks, nacc = verify_ref(p_logits, d, torch.tensor([1.0]), torch.tensor([0], dtype=torch.int32),
                            torch.tensor([1.0]), torch.tensor([1], dtype=torch.int64), torch.tensor([0]),
                            torch.tensor([0], dtype=torch.int64), draft_probs=q[None])
    assert int(nacc[0]) == 2 and toks[0, :2].tolist() == [1, 3]


@pytest.fixture(scope="module")
def peaked_model():
    # a tiny decoder whose next-token distributions are peaked enough for a chi-square test
    cfg = get_config("tiny-llama").replace(init_std=0.25)
    return cfg, prepare_weights(cfg, "cpu", seed=0, max_pos=64)


def test_speculative_sampling_matches_plain_sampling(peaked_model):
    """Second and third tokens of one prompt over many request seeds: a draft model (the same
    weights, sampled at temperature 1.5 against the target's 0.7, so p != q) with gamma 2, versus
    plain sampling; two-sample chi-square on the token counts."""
    cfg, mw = peaked_model
    prompt = [5, 17, 99, 3]
    n = 1200
    sp = [SamplingParams(max_tokens=3, temperature=0.7, seed=s) for s in range(n)]

    def run(spec: bool):
        out = []
        for b in range(0, n, 16):
            runner = ModelRunner(mw, max_batch=16, max_seq_len=32)
            spec_cfg = None
            if spec:
                drunner = ModelRunner(mw, max_batch=16, max_seq_len=32)
                spec_cfg = SpecConfig(gamma=2, drafter=DraftModelDrafter(drunner, temperature=1.5))
            eng = LLMEngine(runner, spec=spec_cfg)
            out += eng.generate([prompt] * len(sp[b:b + 16]), sp[b:b + 16])
            if spec:
                assert eng.stats["spec_drafted"] > 0
        return out

    plain, specd = run(False), run(True)
    for pos in (1, 2):
        a = np.bincount([o[pos] for o in plain], minlength=cfg.vocab)
        b = np.bincount([o[pos] for o in specd], minlength=cfg.vocab)
        keep = (a + b) >= 10
        table = np.stack([np.append(a[keep], a[~keep].sum()), np.append(b[keep], b[~keep].sum())])
        table = table[:, table.sum(0) > 0]
        assert scipy_stats.chi2_contingency(table).pvalue > 1e-3, pos
