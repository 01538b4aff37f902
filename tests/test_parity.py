"""Parity harness on CPU: the engine, teacher-forced, agrees with the naive f32 reference at
every position (top-1 and KL), for the dense, Qwen2-variant and MoE tiny models; the report
detects a perturbed model."""
import torch

from syntropy_b200.bench.parity import fidelity, gate, run


def test_engine_matches_reference_teacher_forced():
    for model in ("tiny-llama", "tiny-qwen2", "tiny-qwen-moe"):
        rep = run(model, 24, "cpu", seed=3)
        assert rep["positions"] == 23
        assert rep["top1_agreement"] == 1.0 and rep["kl_mean"] < 1e-6 and rep["gate"], rep


def test_report_detects_disagreement():
    g = torch.Generator().manual_seed(0)
    ref = torch.randn(16, 50, generator=g)
    assert gate(fidelity(ref.clone(), ref), "fp32")
    noisy = fidelity(ref + torch.randn(16, 50, generator=g), ref)
    assert noisy["top1_agreement"] < 1.0 and noisy["kl_mean"] > 1e-2 and not gate(noisy, "q4")
