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


def test_planner_prices_from_a_probe_report():
    """The hardware model follows a probe report: a slower host link moves more of the host
    tier to the CPU, a faster CPU pool likewise, and the predicted step follows the numbers."""
    from syntropy_b200.models.config import get_config
    from syntropy_b200.planner.planner import HardwareModel, best_cpu_share, plan_placement
    base = {"gpu": {"hbm_copy_gbs": 6448.4, "h2d_gbs": 55.0, "graph_kernel_gap_us": 1.1, "mem_gb": 183.4},
            "host": {"cpu_expert_gbs": 67.0}}
    hw = HardwareModel.from_probe(base)
    assert hw.hbm_gbs == 6448.4 and hw.pcie_gbs == 55.0 and hw.launch_gap_us == 1.1
    slow_link = HardwareModel.from_probe({**base, "gpu": {**base["gpu"], "h2d_gbs": 20.0}})
    fast_cpu = HardwareModel.from_probe({**base, "host": {"cpu_expert_gbs": 150.0}})
    assert best_cpu_share(slow_link) > best_cpu_share(hw) < best_cpu_share(fast_cpu)
    cfg = get_config("qwen3-235b-a22b")
    p0 = plan_placement(cfg, 1, 32, 1024, cache_frac=0.6, hw=hw)
    p1 = plan_placement(cfg, 1, 32, 1024, cache_frac=0.6, hw=slow_link)
    assert p1.predicted_step_ms > p0.predicted_step_ms and p1.cpu_expert_share > p0.cpu_expert_share


def test_cpu_expert_probe_reports_a_rate():
    from syntropy_b200._ext import ext
    from syntropy_b200.probe import probe_cpu_experts
    r = probe_cpu_experts(threads=2, seconds=0.4)
    if ext().cpu_simd_available():
        assert r["cpu_expert_gbs_per_thread"] > 0 and r["cpu_expert_gbs"] > 0 and r["cpu_read_gbs"] > 0
