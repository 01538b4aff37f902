"""Cost-model placement planner (reference: crates/solver; plan/rfcs/RFC-0011)."""
from .planner import HardwareModel, plan_placement  # noqa: F401
