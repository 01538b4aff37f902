"""Saved sessions: a sequence saved mid-generation and restored into a fresh engine over the
same model continues with exactly the tokens of an uninterrupted run (no re-prefill)."""
import torch

from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def test_save_restore_continues_exactly():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, "cpu", state_dict=synthetic_state_dict(cfg, seed=2))
    prompt = torch.randint(0, cfg.vocab, (21,), generator=torch.Generator().manual_seed(4)).tolist()
    sp = SamplingParams(max_tokens=12, temperature=0.8, seed=5)
    want = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=64)).generate([prompt], sp)[0]

    eng = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=64))
    sid = eng.add_request(prompt, sp)
    for _ in range(6):  # prefill + 5 decode steps
        eng.step()
    state = eng.save_session(sid)
    assert len(state["output"]) == 6

    eng2 = LLMEngine(ModelRunner(mw, max_batch=2, max_seq_len=64))
    sid2 = eng2.restore_session(state)
    while eng2.has_work():
        eng2.step()
    got = eng2.finished[sid2].output
    assert got == want


def test_expert_profile_persists(tmp_path):
    from syntropy_b200.experts.cache import ExpertStats
    st = ExpertStats(3, 8)
    st.observe(1, torch.tensor([0, 4, 0, 1, 0, 0, 9, 0]))
    p = str(tmp_path / "experts.pt")
    st.save(p, model="tiny-qwen-moe")
    st2 = ExpertStats.load(p, model="tiny-qwen-moe")
    assert torch.equal(st2.score, st.score) and torch.equal(st2.total, st.total)
    import pytest
    with pytest.raises(ValueError):
        ExpertStats.load(p, model="other")
