"""Router-predicted expert prefetch during decode (VRAM cap with a pinned host tier): tokens
equal the same engine without prefetch (the GEMVs read byte-identical weights, from the
staging copies instead of host memory), with CUDA graphs; after a step the pointer tables
of a predicted host expert point into the VRAM staging bank."""
import pytest
import torch

from syntropy_b200.experts.cache import ExpertCache
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

pytestmark = pytest.mark.gpu


def _run(cuda, prefetch, rebalance_every=64, want_runner=False):
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=21)
    cache = ExpertCache(mw.layers, 0.5, cuda)
    if prefetch:
        assert cache.enable_decode_prefetch(cfg.n_experts)
    runner = ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=True)
    runner.expert_cache = cache
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (17, 40, 5, 64)]
    outs = LLMEngine(runner, rebalance_every=rebalance_every).generate(prompts, SamplingParams(max_tokens=8))
    return (outs, cache, runner) if want_runner else (outs, cache)


def test_prefetch_matches_and_stages(cuda):
    want, _ = _run(cuda, False)
    got, cache = _run(cuda, True)
    assert got == want
    torch.cuda.synchronize()
    # the second MoE layer's table: some predicted host expert now points into staging
    L = cache.layers[1]
    b = L.expert_tier
    st = cache._staging[1][0]["q"]
    lo, hi = st.data_ptr(), st.data_ptr() + st.numel() * st.element_size()
    live = L.experts_gu.qw_ptrs.cpu().tolist()
    staged = [e for e in range(b.E) if b.slot_of[e] < 0 and lo <= live[e] < hi]
    assert staged, "no predicted host expert was staged"
    pred = b.pred.cpu().tolist()
    assert all(pred[b.e0 + e] for e in staged)


def test_adaptation_between_graph_steps(cuda):
    """Residency adapts every 2 decode steps (weights swapped, pointer tables rewritten in
    place under the captured graphs): tokens do not change, and the routing kernels counted
    every routed pair (prefill rows + decode rows, top_k each)."""
    want, _ = _run(cuda, False)
    got, cache, runner = _run(cuda, True, rebalance_every=2, want_runner=True)
    assert got == want
    st = runner.expert_stats
    assert st is not None
    k = runner.cfg.top_k
    n_rows = (17 + 40 + 5 + 64) + 4 * 7  # prefill rows, then 7 decode steps of 4 rows
    left = runner.route_counts.sum(1).cpu()  # counts since the last adaptation
    for li, L in enumerate(cache.layers):
        i = runner._layer_index[id(L)]
        assert int(st.total[li].sum()) + int(left[i]) == n_rows * k
    assert any(b.slot_of != list(range(b.n_res)) + [-1] * (b.E - b.n_res) for b in cache.banks), "no swap happened"


def _run_bulk(cuda, cpu_share=0.0, rebalance_every=64):
    from syntropy_b200.experts.cpu_tier import CpuExpertTier
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=21)
    cache = ExpertCache(mw.layers, 0.5, cuda)
    runner = ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=True)
    runner.expert_cache = cache
    # the BF16 family: exact products, so the tokens must equal the GPU-only engine (the int16
    # family rounds activations to 16 bits per block and may flip a near-tie; its error is
    # checked against the f32 product in test_cpu_experts.py)
    tier = CpuExpertTier(cache, cfg, max_rows=runner.max_batch, cpu_share=cpu_share, threads=4, mode=1) \
        if cpu_share else None
    assert cache.enable_decode_staging()
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (17, 40, 5, 64)]
    try:
        outs = LLMEngine(runner, rebalance_every=rebalance_every).generate(prompts, SamplingParams(max_tokens=8))
    finally:
        if tier is not None:
            tier.close()
    return outs, cache


@pytest.mark.parametrize("cpu_share,rebalance_every", [(0.0, 64), (0.5, 64), (0.5, 2)])
def test_bulk_staging_matches(cuda, cpu_share, rebalance_every):
    """Bulk DMA staging of every GPU-read host expert (double-buffered across layers, captured
    in the decode graphs), alone, beside the CPU tier, and across residency swaps every two
    steps: tokens equal the engine without staging; the live tables of GPU-read host experts
    point into the layer's staging bank, the CPU's experts stay null."""
    want, _ = _run(cuda, False)
    got, cache = _run_bulk(cuda, cpu_share, rebalance_every)
    assert got == want
    for li, L in enumerate(cache.layers):
        b = L.expert_tier
        st = cache._staging[li % 2][0]["q"]
        lo, hi = st.data_ptr(), st.data_ptr() + st.numel() * st.element_size()
        live = L.experts_gu.qw_ptrs.cpu().tolist()
        for e in range(b.E):
            if e in b.cpu_owned:
                assert live[e] == 0
            elif b.slot_of[e] < 0:
                assert lo <= live[e] < hi
        assert sorted(b.host_of[e] for e in b.cpu_owned) == list(range(len(b.cpu_owned)))


def test_host_tier_pack_round_trip(cuda, tmp_path):
    """The pinned host tier saves to a pack and reloads through the native I/O pool (direct
    reads into aligned bounce buffers); tokens afterwards equal the engine's before."""
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=21)
    cache = ExpertCache(mw.layers, 0.5, cuda)
    p = str(tmp_path / "tier.pack")
    cache.save_host_tier(p)
    want = [p_["qh"].clone() for b in cache.banks for p_ in b.parts if p_ is not None]
    for b in cache.banks:
        for p_ in b.parts:
            if p_ is not None:
                p_["qh"].zero_()
                p_["sh"].zero_()
    assert cache.load_host_tier(p, threads=4) > 0
    got = [p_["qh"] for b in cache.banks for p_ in b.parts if p_ is not None]
    assert all(torch.equal(a, b) for a, b in zip(want, got))
    runner = ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=True)
    runner.expert_cache = cache
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (17, 40, 5, 64)]
    assert LLMEngine(runner).generate(prompts, SamplingParams(max_tokens=8)) == _run(cuda, False)[0]


def test_prefill_over_two_banks_matches_resident(cuda):
    """Prefill with half the experts in the host tier: the grouped GEMMs stream the residents
    and the staged host experts from two contiguous banks through TMA (per-expert bank
    selector); the last-token logits equal those of the same model with every expert resident
    (one contiguous bank)."""
    cfg = get_config("small-qwen-moe")
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, cfg.vocab, (200,), generator=g)
    blocks = list(range(1, 1 + (200 + 15) // 16))
    slots = torch.tensor([blocks[p // 16] * 16 + p % 16 for p in range(200)])

    def logits(capped):
        mw = prepare_weights(cfg, cuda, seed=21)
        runner = ModelRunner(mw, max_batch=4, max_seq_len=256)
        if capped:
            runner.expert_cache = ExpertCache(mw.layers, 0.5, cuda)
        out = runner.prefill(prompt, torch.arange(200), slots, [0, 200], block_lists=[blocks])[0].float().cpu()
        torch.cuda.synchronize()
        return out, runner
    want, _ = logits(False)
    got, runner = logits(True)
    assert runner.expert_cache.staged_banks(runner.mw.layers[-1]) is not None
    assert ((got - want).norm() / want.norm()).item() < 1e-4
