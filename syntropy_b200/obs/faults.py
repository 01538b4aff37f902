"""Fault injection points (host side only).

`fault_point("area.component.op")` is a no-op unless a plan is installed (programmatically
or from SYN_FAULT_PLAN, a JSON list).  A rule matches a point name and fires on the n-th
hit (`nth`) or with probability `p` from a seeded generator; effects: "error" (raise
SynError), "delay" (sleep), "drop" (return True so the caller drops the message), "exit"
(terminate the process: a rank that dies between steps).  Device-side faults are not built
(a GPU fault on a shared pool is never provoked on purpose).
Reference: crates/obs/src/faults.rs:1-129, crates/obs/src/faults/inject.rs:24-40.
"""
from __future__ import annotations

import json
import os
import random
import threading
import time
from dataclasses import dataclass, field

from ..core.errors import ErrorClass, SynError


@dataclass
class FaultRule:
    point: str
    effect: str = "error"        # error | delay | drop | exit
    nth: int | None = None       # fire on this hit (1-based)
    p: float | None = None       # or with this probability
    seed: int = 0
    delay_s: float = 0.0
    error_class: str = "transient"
    hits: int = 0
    fired: int = 0
    _rng: random.Random = field(default=None, repr=False)

    def should_fire(self) -> bool:
        self.hits += 1
        if self.nth is not None:
            return self.hits == self.nth
        if self.p is not None:
            if self._rng is None:
                self._rng = random.Random(self.seed)
            return self._rng.random() < self.p
        return True


class FaultPlan:
    def __init__(self, rules: list[FaultRule]):
        self.rules = rules
        self._lock = threading.Lock()

    @classmethod
    def from_json(cls, text: str) -> "FaultPlan":
        return cls([FaultRule(**r) for r in json.loads(text)])

    def check(self, point: str) -> bool:
        with self._lock:
            for r in self.rules:
                if r.point == point or (r.point.endswith("*") and point.startswith(r.point[:-1])):
                    if r.should_fire():
                        r.fired += 1
                        return self._apply(r, point)
        return False

    def _apply(self, r: FaultRule, point: str) -> bool:
        if r.effect == "delay":
            time.sleep(r.delay_s)
            return False
        if r.effect == "drop":
            return True
        if r.effect == "exit":
            os._exit(17)
        raise SynError(ErrorClass(r.error_class), f"injected fault at {point}")


_PLAN: FaultPlan | None = None
if os.environ.get("SYN_FAULT_PLAN"):
    _PLAN = FaultPlan.from_json(os.environ["SYN_FAULT_PLAN"])


def install(plan: FaultPlan | None):
    global _PLAN
    _PLAN = plan


def fault_point(point: str) -> bool:
    """Returns True when the caller should drop the current message."""
    return _PLAN.check(point) if _PLAN is not None else False
