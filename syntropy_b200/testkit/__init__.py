"""Test kit: deterministic simulation on virtual time (sim.py) and scripted runners for
supervisor and cluster logic (reference crates/testkit)."""
from .sim import LinkModel, SimFabric, SimWorld  # noqa: F401
