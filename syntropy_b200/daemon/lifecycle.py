"""Runner lifecycle: Fetching -> Packing -> Loading -> Warming -> Ready -> Draining ->
Stopped, with Failed reachable from any state (reference: crates/runner/src/lifecycle.rs:
38-199).  Transitions are validated; each records its time for the bring-up report."""
from __future__ import annotations

import enum
import time


class LifecycleState(enum.Enum):
    FETCHING = "fetching"
    PACKING = "packing"
    LOADING = "loading"
    WARMING = "warming"
    READY = "ready"
    DRAINING = "draining"
    STOPPED = "stopped"
    FAILED = "failed"


_NEXT = {
    LifecycleState.FETCHING: {LifecycleState.PACKING, LifecycleState.LOADING},
    LifecycleState.PACKING: {LifecycleState.LOADING},
    LifecycleState.LOADING: {LifecycleState.WARMING},
    LifecycleState.WARMING: {LifecycleState.READY},
    LifecycleState.READY: {LifecycleState.DRAINING},
    LifecycleState.DRAINING: {LifecycleState.STOPPED},
    LifecycleState.STOPPED: set(),
    LifecycleState.FAILED: set(),
}


class Lifecycle:
    def __init__(self, clock=time.monotonic):
        self.clock = clock
        self.state = LifecycleState.FETCHING
        self.history = [(self.state, clock())]
        self.error: str | None = None

    def to(self, new: LifecycleState, error: str | None = None):
        if new == LifecycleState.FAILED:
            self.error = error or "failed"
        elif new not in _NEXT[self.state]:
            raise ValueError(f"illegal lifecycle transition {self.state.value} -> {new.value}")
        self.state = new
        self.history.append((new, self.clock()))

    @property
    def ready(self) -> bool:
        return self.state == LifecycleState.READY

    def durations(self) -> dict:
        out = {}
        for (s, t0), (_, t1) in zip(self.history, self.history[1:]):
            out[s.value] = out.get(s.value, 0.0) + (t1 - t0)
        return out
