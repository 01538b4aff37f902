"""MoE expert residency: VRAM expert cache over a pinned host-RAM tier, routing statistics
with decayed-LFU ranking, and the deterministic hit/copy/CPU split rule."""
from .cache import ExpertCache, ExpertStats  # noqa: F401
