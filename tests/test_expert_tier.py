"""Expert cache residency on CPU tensors: the decayed-LFU planner (native) swaps the coldest
residents for the hottest host experts, every expert's weights survive the swaps byte for
byte, and the pointer tables point at each expert's current home."""
from types import SimpleNamespace

import torch

from syntropy_b200.experts.cache import ExpertCache, ExpertStats


def _bank(E, g):
    return SimpleNamespace(qw=torch.randint(-2**31, 2**31 - 1, (E, 4, 32), dtype=torch.int32, generator=g),
                           sm=torch.randn(E, 4, 8, generator=g).half(), E=E, e0=0, qw_ptrs=None, sm_ptrs=None,
                           bank_contiguous=True)


def test_rebalance_swaps_and_keeps_weights():
    g = torch.Generator().manual_seed(0)
    E = 8
    gu, dn = _bank(E, g), _bank(E, g)
    orig = [(gu.qw[e].clone(), gu.sm[e].clone(), dn.qw[e].clone(), dn.sm[e].clone()) for e in range(E)]
    layer = SimpleNamespace(is_moe=True, experts_gu=gu, experts_down=dn)
    cache = ExpertCache([layer], 0.5, torch.device("cpu"))
    b = cache.banks[0]
    assert b.n_res == 4 and [s >= 0 for s in b.slot_of] == [True] * 4 + [False] * 4
    st = ExpertStats(1, E)
    st.observe(0, torch.tensor([5, 0, 9, 1, 8, 0, 0, 7]))
    n = cache.rebalance(st, max_swaps_per_layer=4)
    # cold residents 1 (0), 3 (1) leave for hot host experts 4 (8), 7 (7); 0 (5) vs 5/6 (0) stays
    assert n == 2
    assert b.resident_mask().tolist() == [True, False, True, False, True, False, False, True]
    for e in range(E):
        q, s = b.weight_of(0, e)
        assert torch.equal(q, orig[e][0]) and torch.equal(s, orig[e][1])
        q, s = b.weight_of(1, e)
        assert torch.equal(q, orig[e][2]) and torch.equal(s, orig[e][3])
        assert int(gu.qw_ptrs[e]) == b.weight_of(0, e)[0].data_ptr()
        assert int(dn.sm_ptrs[e]) == b.weight_of(1, e)[1].data_ptr()
    # a second pass with the same scores finds nothing worth moving
    assert cache.rebalance(st, max_swaps_per_layer=4) == 0


def test_cpu_tier_split_and_detach():
    """The CPU tier takes its share of each layer's host experts (null GPU pointers for them),
    follows residency changes, and hands everything back on detach."""
    from syntropy_b200.experts.cpu_tier import CpuExpertTier
    g = torch.Generator().manual_seed(1)
    E = 8
    gu, dn = _bank(E, g), _bank(E, g)
    layer = SimpleNamespace(is_moe=True, experts_gu=gu, experts_down=dn)
    cache = ExpertCache([layer], 0.5, torch.device("cpu"))
    cfg = SimpleNamespace(n_experts=E, top_k=2, hidden=256, moe_ffn=128)
    tier = CpuExpertTier(cache, cfg, max_rows=4, cpu_share=0.5, threads=2, cpus=[])
    try:
        b = cache.banks[0]
        assert cache.cpu_tier is tier and b.cpu_owned == {4, 5}  # half of host experts 4..7
        ptrs = gu.qw_ptrs.tolist()
        assert [p == 0 for p in ptrs] == [False] * 4 + [True, True, False, False]
        st = ExpertStats(1, E)
        st.observe(0, torch.tensor([0, 9, 9, 9, 9, 0, 0, 0]))
        assert cache.rebalance(st, max_swaps_per_layer=1) == 1  # expert 4 comes in for expert 0
        assert b.slot_of[4] >= 0 and b.cpu_owned == {0, 5}
        assert int(gu.qw_ptrs[4]) != 0 and int(gu.qw_ptrs[0]) == 0
        tier.detach()
        assert cache.cpu_tier is None and not b.cpu_owned
        assert all(int(p) != 0 for p in gu.qw_ptrs) and all(int(p) != 0 for p in dn.sm_ptrs)
    finally:
        tier.close()


def test_adapt_experts_reports_the_window_hit_rate():
    """The runner's rebalance folds the window's routing counts into the scores and records the
    share of routed pairs whose expert was in VRAM during that window."""
    from syntropy_b200.runtime.runner import ModelRunner
    g = torch.Generator().manual_seed(0)
    E = 8
    layer = SimpleNamespace(is_moe=True, experts_gu=_bank(E, g), experts_down=_bank(E, g))
    cache = ExpertCache([layer], 0.5, torch.device("cpu"))
    counts = torch.tensor([[5, 0, 9, 1, 8, 0, 0, 7]], dtype=torch.int32)  # residents: experts 0-3
    fake = SimpleNamespace(expert_cache=cache, route_counts=counts.clone(), expert_stats=None, ep=None,
                           cfg=SimpleNamespace(n_experts=E), _layer_index={id(layer): 0}, expert_hit_rate=None)
    assert ModelRunner.adapt_experts(fake, max_swaps_per_layer=4) == 2
    assert abs(fake.expert_hit_rate - 15 / 30) < 1e-9
    assert int(fake.route_counts.sum()) == 0  # the window's counts were consumed
