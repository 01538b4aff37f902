"""KV tiering by preemption on CPU: with a page pool too small for every running sequence to
grow, the engine swaps the newest sequences' KV pages out to host memory and back in later;
the tokens equal a run with an ample pool."""
import pytest
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


def test_swap_with_prefix_cache():
    """Shared prefix pages (refcounted) survive a preemption of one of their users; cached
    prefixes nobody uses are evicted before any running sequence is preempted."""
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=2)
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, cfg.vocab, (32,), generator=g).tolist()
    prompts = [shared + torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (3, 9, 5)]
    params = SamplingParams(max_tokens=30)
    want = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(prompts, params)
    for nb in (8, 9, 10, 12):  # 8 and 9 once left a preempted sequence behind unreferenced cached pages
        eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, num_blocks=nb), prefix_cache=True)
        for p in prompts:
            eng.add_request(p, params)
        for _ in range(500):  # bounded: a scheduling livelock fails instead of hanging
            if not eng.has_work():
                break
            eng.step()
        assert not eng.has_work(), (nb, len(eng.running), len(eng.waiting), len(eng.swapped))
        got = [eng.finished[i].output for i in sorted(eng.finished)]
        assert got == want, nb
        assert eng.stats["swapped_out"] == eng.stats["swapped_in"]


def test_request_larger_than_the_pool_is_rejected():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=2)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, num_blocks=3))
    with pytest.raises(ValueError, match="KV pages"):
        eng.add_request(list(range(5, 65)), SamplingParams(max_tokens=4))
    eng.add_request(list(range(5, 20)), SamplingParams(max_tokens=4))  # fits: served
    while eng.has_work():
        eng.step()


@pytest.mark.parametrize("host_budget", [0, 6000])
def test_swap_spills_to_files_past_the_host_budget(tmp_path, host_budget):
    """A host budget below the preempted pages sends them to pack files (budget 0: all of them;
    a small budget: the tail of the queue) and back; tokens equal the ample-pool run and no
    file is left behind."""
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=2)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (20, 14, 30, 9)]
    params = SamplingParams(max_tokens=40)
    want = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(prompts, params)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, num_blocks=9), kv_host_bytes=host_budget,
                    kv_spill_dir=str(tmp_path / "kv"))
    assert eng.generate(prompts, params) == want
    st = eng.kv_store.stats
    assert eng.stats["swapped_out"] > 0 and st["spilled"] > 0 and st["restored"] == st["spilled"]
    assert eng.kv_store.host_bytes == 0 and eng.kv_store.disk_bytes == 0
    assert not list((tmp_path / "kv").iterdir())


def test_swap_store_tiers_and_digest(tmp_path):
    from syntropy_b200.kv.tiers import SwapStore
    a = [torch.randn(3, 4, 16).to(torch.bfloat16) for _ in range(2)]
    b = [torch.randn(2, 4, 16).to(torch.bfloat16) for _ in range(2)]
    nb_a = sum(t.numel() * 2 for t in a)
    st = SwapStore(host_budget=nb_a, spill_dir=str(tmp_path))
    ea, eb = st.put(1, [t.clone() for t in a]), st.put(2, [t.clone() for t in b])
    assert st.where(ea) == "host" and st.where(eb) == "disk"
    assert all(torch.equal(x, y) for x, y in zip(st.take(ea), a))
    st.refill([eb])  # room again: the next to resume comes back into RAM
    assert st.where(eb) == "host" and not list(tmp_path.glob("*.pack"))
    assert all(torch.equal(x, y) for x, y in zip(st.take(eb), b))
    # a damaged spill file is caught by its digest, not handed back as KV
    st2 = SwapStore(host_budget=0, spill_dir=str(tmp_path))
    ec = st2.put(3, [t.clone() for t in b])
    with open(ec.path, "r+b") as f:
        f.seek(5)
        f.write(b"\xff\xfe")
    with pytest.raises(ValueError, match="digest"):
        st2.take(ec)
    st2.drop(ec)
    assert not list(tmp_path.glob("*.pack*"))


def test_failed_spill_keeps_the_sequence_running(tmp_path, monkeypatch):
    """A spill that cannot be written raises from the step, and the sequence it was preempting
    still holds its pages and runs (nothing is lost)."""
    from syntropy_b200.kv import tiers
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=2)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (20, 14, 30, 9)]
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, num_blocks=9), kv_host_bytes=0,
                    kv_spill_dir=str(tmp_path / "kv"))

    def broken(*a, **k):
        raise OSError(28, "No space left on device")
    monkeypatch.setattr(tiers.SwapStore, "_spill", broken)
    for p in prompts:
        eng.add_request(p, SamplingParams(max_tokens=40))
    with pytest.raises(OSError):
        for _ in range(200):
            if not eng.has_work():
                break
            eng.step()
    assert not eng.swapped and eng.kv_store.host_bytes == 0
    assert all(s.blocks for s in eng.running)  # every running sequence still holds its pages
