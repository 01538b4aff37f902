"""Placement plans: how a model instance maps onto devices (reference: crates/core/src/
plan.rs, crates/core/src/plan/stage.rs:54-130, crates/core/src/plan/speculative.rs)."""
from __future__ import annotations

import enum
from dataclasses import dataclass, field


class CollectiveAlgo(enum.Enum):
    ONE_SHOT = "one_shot"      # every member reads every partial, sums in member order
    RING = "ring"              # reduce-scatter then all-gather
    NCCL = "nccl"              # library collective (the baseline)
    FUSED = "fused"            # compute + collective in one kernel over peer memory


@dataclass
class TpSplit:
    """How a layer's work divides over TP members (whole KV heads; weights by fraction)."""
    fractions: list[float]
    kv_heads: list[int] | None = None
    experts_tp: bool = False  # split each expert like the dense FFN (TP inside experts)


@dataclass
class ExpertOwnerMap:
    """Expert e of layer l is owned by member owner[l][e] (expert parallelism)."""
    owner: list[list[int]]

    @classmethod
    def contiguous(cls, n_layers: int, n_experts: int, n_members: int) -> "ExpertOwnerMap":
        per = n_experts // n_members
        return cls([[e // per for e in range(n_experts)] for _ in range(n_layers)])

    def local_range(self, layer: int, member: int) -> tuple[int, int]:
        own = [e for e, m in enumerate(self.owner[layer]) if m == member]
        return (own[0], own[-1] + 1) if own else (0, 0)


class ParallelismMode(enum.Enum):
    LOCAL = "local"                  # one device
    INTRA_NODE_TP = "intra_node_tp"  # tensor parallel over NVLink
    EP = "ep"                        # expert parallel (+ data-parallel attention)
    PP = "pp"                        # pipeline stages over NCCL p2p
    DP = "dp"                        # independent replicas


@dataclass
class StagePlan:
    layers: tuple[int, int]          # [first, last) layer of the stage
    devices: list[int]
    mode: ParallelismMode = ParallelismMode.LOCAL
    tp: TpSplit | None = None
    experts: ExpertOwnerMap | None = None
    collective: CollectiveAlgo = CollectiveAlgo.FUSED


class DraftSource(enum.Enum):
    MTP = "mtp"
    DRAFT_HEAD = "draft_head"
    DRAFT_MODEL = "draft_model"
    PROMPT_LOOKUP = "prompt_lookup"


class Acceptance(enum.Enum):
    EXACT = "exact"  # distribution-preserving (greedy / point-mass / residual)


@dataclass
class SpeculativeConfig:
    source: DraftSource = DraftSource.MTP
    gamma: int = 1                   # drafted tokens per step
    acceptance: Acceptance = Acceptance.EXACT


@dataclass
class PlacementPlan:
    model: str
    stages: list[StagePlan]
    expert_cache_frac: float = 1.0   # VRAM-resident share of each rank's experts
    kv_pages: int = 0
    max_batch: int = 64
    speculative: SpeculativeConfig | None = None
    predicted_step_ms: float | None = None
    cost_terms: dict = field(default_factory=dict)
    cpu_expert_share: float = 0.0    # share of the host experts computed by host CPU threads

    @property
    def n_devices(self) -> int:
        return len({d for s in self.stages for d in s.devices})

    def describe(self) -> str:
        lines = [f"plan for {self.model}: {self.n_devices} device(s)"]
        for s in self.stages:
            lines.append(f"  layers {s.layers[0]}..{s.layers[1]} on {s.devices} mode={s.mode.value} "
                         f"collective={s.collective.value}")
        if self.expert_cache_frac < 1.0:
            lines.append(f"  expert cache: {self.expert_cache_frac:.0%} of experts VRAM-resident, rest in pinned host RAM")
            if self.cpu_expert_share > 0:
                lines.append(f"  host tier: {self.cpu_expert_share:.0%} of the host experts computed by host CPU "
                             f"threads, the rest read over PCIe (concurrently)")
        if self.predicted_step_ms is not None:
            lines.append(f"  predicted decode step: {self.predicted_step_ms:.2f} ms")
            for k, v in sorted(self.cost_terms.items()):
                lines.append(f"    {k:>24}: {v:.3f} ms")
        return "\n".join(lines)
