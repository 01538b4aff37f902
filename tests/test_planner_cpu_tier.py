"""Planner with the host CPU tier: on one GPU with a VRAM cap the host experts are split
between PCIe reads and CPU threads at the share that balances the two concurrent paths, and the
plan predicts a shorter step than PCIe alone; under expert parallelism no CPU share is planned."""
from syntropy_b200.core.plan import ParallelismMode
from syntropy_b200.models.config import get_config
from syntropy_b200.planner import plan_placement
from syntropy_b200.planner.planner import HardwareModel, best_cpu_share, price_decode


def test_cpu_share_balances_paths():
    hw = HardwareModel()
    cfg = get_config("qwen3-235b-a22b")
    s = best_cpu_share(hw)
    assert 0.5 < s < 0.8
    t = {x: price_decode(cfg, 1, 32, 1280, ParallelismMode.LOCAL, 0.6, hw, cpu_share=x)["total"]
         for x in (0.3, s, 0.95)}
    assert t[s] < t[0.3] and t[s] < t[0.95]


def test_plan_uses_cpu_tier_on_one_gpu_only():
    cfg = get_config("qwen3-235b-a22b")
    with_cpu = plan_placement(cfg, 1, 32, 1280, cache_frac=0.6, hw=HardwareModel())
    without = plan_placement(cfg, 1, 32, 1280, cache_frac=0.6, hw=HardwareModel(), cpu_tier=False)
    assert with_cpu.cpu_expert_share > 0 and without.cpu_expert_share == 0
    assert with_cpu.predicted_step_ms < without.predicted_step_ms
    assert "host CPU threads" in with_cpu.describe()
    ep8 = plan_placement(cfg, 8, 32, 1280, cache_frac=0.6, hw=HardwareModel())
    assert ep8.cpu_expert_share == 0
