"""Cost-model planner: picks tensor / expert / pipeline parallelism and the expert-cache
share for 1, 2, 4 or 8 B200s, pricing each candidate's decode step from measured
bandwidths.

Decode is priced term by term (the reference's CostTerm idea, crates/obs/src/cost_term.rs):
  weights  = bytes streamed per step / (HBM bandwidth * kernel efficiency)
  kv       = KV bytes read per step / HBM bandwidth
  host     = cold-expert bytes split between the GPU's PCIe reads and the host CPU threads,
             which run concurrently: max(PCIe part / PCIe rate, CPU part / CPU rate) plus the
             per-layer hand-off cost; the planner picks the CPU share that balances the two
             paths (one GPU per host slice)
  collect  = per-layer collective latency (alpha) + bytes / NVLink bandwidth (beta)
  launch   = kernels per step * graph-launch gap
The collective model follows crates/solver/src/collective.rs:236-333 (one-shot vs ring).
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass

from ..core.plan import CollectiveAlgo, ExpertOwnerMap, ParallelismMode, PlacementPlan, StagePlan, TpSplit
from ..models.config import ModelConfig


@dataclass
class HardwareModel:
    hbm_gbs: float = 6446.6        # measured copy bandwidth
    hbm_eff: float = 0.55          # achieved fraction for 4-bit GEMV streams (measured)
    nvlink_gbs: float = 770.0      # peer copy per direction
    nvlink_alpha_us: float = 6.0   # one fused flag round trip
    nccl_alpha_us: float = 18.0    # small NCCL collective latency
    pcie_gbs: float = 55.5         # pinned H2D (measured on the B200 box)
    # host tier with the CPU expert pool: per-layer time = fixed + max(PCIe part, CPU part); the
    # PCIe rate fitted to capped Qwen3 decode on one B200 node slice, the CPU rate to the measured
    # balance of the int16 VNNI pool (share 0.7 against the link: 0.7 / 0.3 x 50 GB/s)
    pcie_read_gbs: float = 50.0    # GPU reading host experts in place while the CPU also reads DRAM
    cpu_expert_gbs: float = 117.0  # host CPU expert pool, 14 threads
    cpu_tier_layer_ms: float = 2.7  # per MoE layer: hand-off, collect and the serial part around them
    vram_gb: float = 178.0
    launch_gap_us: float = 1.2     # per kernel inside a CUDA graph
    tflops: float = 1422.0         # sustained bf16

    @classmethod
    def from_probe(cls, probe: dict, base: "HardwareModel | None" = None) -> "HardwareModel":
        """Prices from a probe report (`python -m syntropy_b200 probe --full --out FILE`): HBM copy,
        pinned host-to-device and peer copy bandwidths, peer round-trip latency, the CUDA-graph
        kernel gap, and the host CPU expert pool's rate.  Missing probes keep the base value
        (the defaults above, measured on a B200 node)."""
        hw = base or cls()
        g = probe.get("gpu", {}) or {}
        h = probe.get("host", {}) or {}
        if g.get("hbm_copy_gbs"):
            hw.hbm_gbs = float(g["hbm_copy_gbs"])
        if g.get("h2d_gbs"):
            hw.pcie_gbs = float(g["h2d_gbs"])
            # host experts the GPU reads are staged with the same DMA copies (bulk staging)
            hw.pcie_read_gbs = float(g["h2d_gbs"]) * 0.9
        if g.get("peer_copy_gbs"):
            hw.nvlink_gbs = float(g["peer_copy_gbs"])
        if g.get("peer_latency_us"):
            hw.nvlink_alpha_us = float(g["peer_latency_us"])
        if g.get("graph_kernel_gap_us"):
            hw.launch_gap_us = float(g["graph_kernel_gap_us"])
        if h.get("cpu_expert_gbs"):
            hw.cpu_expert_gbs = float(h["cpu_expert_gbs"])
        if g.get("mem_gb"):
            hw.vram_gb = float(g["mem_gb"]) - 2.0
        return hw

    @classmethod
    def from_measured(cls, path: str | None = None) -> "HardwareModel":
        hw = cls()
        path = path or os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
        try:
            with open(path) as f:
                d = json.load(f)
            hw.hbm_gbs = float(d.get("hbm_gbs", hw.hbm_gbs))
            hw.tflops = float(d.get("bf16_tflops_sustained", hw.tflops))
        except (OSError, ValueError):
            pass
        return hw


def _weight_bytes(cfg: ModelConfig) -> tuple[float, float, float]:
    """(attention+dense bytes per layer, one expert's bytes, lm_head bytes) at 5 bits/weight."""
    bpw = 5.0 / 8 if cfg.weight_quant == "q4" else (1.0 if cfg.weight_quant == "fp8" else 2.0)
    h = cfg.hidden
    attn = (h * (cfg.q_dim + 2 * cfg.kv_dim) + cfg.q_dim * h) * bpw
    expert = 3 * h * cfg.moe_ffn * bpw if cfg.is_moe else 0.0
    head = cfg.vocab * h * bpw
    return attn, expert, head


def best_cpu_share(hw: HardwareModel) -> float:
    """CPU share of the host experts that equalises the two concurrent paths."""
    return hw.cpu_expert_gbs / (hw.cpu_expert_gbs + hw.pcie_read_gbs)


def price_decode(cfg: ModelConfig, n_gpu: int, batch: int, ctx: int, mode: ParallelismMode, cache_frac: float,
                 hw: HardwareModel, fused: bool = True, cpu_share: float = 0.0) -> dict:
    attn_b, exp_b, head_b = _weight_bytes(cfg)
    L = cfg.n_layers
    terms = {}
    if cfg.is_moe:
        E, k = cfg.n_experts, cfg.top_k
        per_rank_tokens = batch / n_gpu if mode == ParallelismMode.EP else batch
        # expected active experts per layer given `batch` tokens routed uniformly
        p_active = 1.0 - (1.0 - k / E) ** batch
        e_local = E / (n_gpu if mode == ParallelismMode.EP else 1)
        active_local = e_local * p_active
        hot = active_local * cache_frac
        cold = active_local * (1.0 - cache_frac)
        attn_rank = attn_b / (n_gpu if mode == ParallelismMode.INTRA_NODE_TP else 1)
        terms["weights"] = L * (hot * exp_b + attn_rank) / (hw.hbm_gbs * 1e9 * hw.hbm_eff) * 1e3
        if cpu_share > 0:
            terms["host_tier"] = L * cold * exp_b * max((1 - cpu_share) / (hw.pcie_read_gbs * 1e9),
                                                        cpu_share / (hw.cpu_expert_gbs * 1e9)) * 1e3
            terms["cpu_handoff"] = L * hw.cpu_tier_layer_ms
        else:
            terms["host_tier"] = L * cold * exp_b / (hw.pcie_gbs * 1e9) * 1e3
        kv_tok = 2 * cfg.kv_dim * 2 * L
        terms["kv"] = per_rank_tokens * ctx * kv_tok / (hw.hbm_gbs * 1e9 * 0.45) * 1e3
        if n_gpu > 1:
            alpha = hw.nvlink_alpha_us if fused else hw.nccl_alpha_us
            msg = per_rank_tokens * cfg.hidden * (2 + 4 * k / n_gpu)
            terms["collectives"] = L * 2 * (alpha * 1e-3 + msg / (hw.nvlink_gbs * 1e9) * 1e3)
        terms["launch"] = L * 11 * hw.launch_gap_us * 1e-3
    else:
        tp = n_gpu if mode == ParallelismMode.INTRA_NODE_TP else 1
        ffn_b = 3 * cfg.hidden * cfg.ffn * (5.0 / 8 if cfg.weight_quant == "q4" else 2.0)
        terms["weights"] = L * (attn_b + ffn_b) / tp / (hw.hbm_gbs * 1e9 * hw.hbm_eff) * 1e3
        kv_tok = 2 * cfg.kv_dim * 2 * L
        terms["kv"] = batch * ctx * kv_tok / tp / (hw.hbm_gbs * 1e9 * 0.45) * 1e3
        if tp > 1:
            alpha = hw.nvlink_alpha_us if fused else hw.nccl_alpha_us
            msg = batch * cfg.hidden * 4
            terms["collectives"] = L * 2 * (alpha * 1e-3 + msg / (hw.nvlink_gbs * 1e9) * 1e3)
        terms["launch"] = L * 8 * hw.launch_gap_us * 1e-3
    terms["lm_head"] = head_b / (hw.hbm_gbs * 1e9 * 0.5) * 1e3
    terms["total"] = sum(v for kk, v in terms.items() if kk != "total")
    return terms


def fits(cfg: ModelConfig, n_gpu: int, mode: ParallelismMode, cache_frac: float, hw: HardwareModel,
         batch: int, ctx: int) -> bool:
    attn_b, exp_b, head_b = _weight_bytes(cfg)
    L = cfg.n_layers
    per_gpu = head_b + 2 * cfg.vocab * cfg.hidden  # head + bf16 embedding
    if cfg.is_moe:
        e_local = cfg.n_experts / (n_gpu if mode == ParallelismMode.EP else 1)
        per_gpu += L * (attn_b + e_local * exp_b * cache_frac)
    else:
        tp = n_gpu if mode == ParallelismMode.INTRA_NODE_TP else 1
        per_gpu += L * (attn_b + 3 * cfg.hidden * cfg.ffn * 5 / 8) / tp
    kv = batch * ctx * 2 * cfg.kv_dim * 2 * L / (n_gpu if mode != ParallelismMode.LOCAL else 1)
    return (per_gpu + kv) / 1e9 < hw.vram_gb * 0.95


def plan_placement(cfg: ModelConfig, n_gpu: int, batch: int = 32, ctx: int = 2048,
                   cache_frac: float | None = None, hw: HardwareModel | None = None,
                   fused: bool = True, cpu_tier: bool = True) -> PlacementPlan:
    hw = hw or HardwareModel.from_measured()
    # the host CPU tier serves one GPU (under expert parallelism each rank reads over PCIe)
    share = best_cpu_share(hw) if cpu_tier and n_gpu == 1 and cfg.is_moe else 0.0
    cands = []
    modes = [ParallelismMode.LOCAL] if n_gpu == 1 else [ParallelismMode.EP, ParallelismMode.INTRA_NODE_TP,
                                                       ParallelismMode.DP]
    if not cfg.is_moe and n_gpu > 1:
        modes = [ParallelismMode.INTRA_NODE_TP, ParallelismMode.DP]
    fracs = [cache_frac] if cache_frac is not None else [1.0, 0.8, 0.6, 0.4]
    for mode in modes:
        for fr in fracs:
            if not fits(cfg, n_gpu, mode, fr, hw, batch, ctx):
                continue
            if mode == ParallelismMode.DP:
                t = price_decode(cfg, 1, max(1, batch // n_gpu), ctx, ParallelismMode.LOCAL, fr, hw)
            else:
                t = price_decode(cfg, n_gpu, batch, ctx, mode, fr, hw, fused, cpu_share=share if fr < 1 else 0.0)
            cands.append((t["total"], mode, fr, t))
    if not cands:
        raise ValueError(f"{cfg.name} does not fit on {n_gpu} GPU(s) at batch {batch}, ctx {ctx}")
    cands.sort(key=lambda c: (c[0], -c[2]))
    total, mode, fr, terms = cands[0]
    devices = list(range(n_gpu))
    stage = StagePlan(layers=(0, cfg.n_layers), devices=devices, mode=mode,
                      collective=CollectiveAlgo.FUSED if fused else CollectiveAlgo.NCCL)
    if mode == ParallelismMode.EP:
        stage.experts = ExpertOwnerMap.contiguous(cfg.n_layers, cfg.n_experts, n_gpu)
    if mode == ParallelismMode.INTRA_NODE_TP:
        stage.tp = TpSplit([1.0 / n_gpu] * n_gpu)
    return PlacementPlan(model=cfg.name, stages=[stage], expert_cache_frac=fr, max_batch=batch,
                         predicted_step_ms=total, cost_terms={k: v for k, v in terms.items() if k != "total"},
                         cpu_expert_share=share if fr < 1 else 0.0)
