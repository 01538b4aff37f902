"""Plain data types shared by every layer: error taxonomy, placement plans, quantisation
schemes, sequences and token frames (reference layer 0: crates/core)."""
from .errors import ErrorClass, SynError  # noqa: F401
from .plan import (  # noqa: F401
    Acceptance, CollectiveAlgo, DraftSource, ExpertOwnerMap, ParallelismMode, PlacementPlan, SpeculativeConfig,
    StagePlan, TpSplit,
)
from .quant import QuantScheme  # noqa: F401
