"""Hash-chained event log and the pure state transition function."""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass, field


@dataclass(frozen=True)
class Event:
    kind: str          # member_join | member_leave | member_suspect | instance_up | instance_down | plan
    term: int
    data: dict

    def encode(self) -> bytes:
        return json.dumps({"kind": self.kind, "term": self.term, "data": self.data}, sort_keys=True).encode()


@dataclass
class ClusterState:
    term: int = 0
    members: dict = field(default_factory=dict)      # node -> {"status": ..., "gpus": n}
    instances: dict = field(default_factory=dict)    # instance -> {"model":..., "plan_epoch":..., "nodes": [...]}
    plan_epoch: int = 0
    applied: int = 0


def apply(state: ClusterState, ev: Event) -> ClusterState:
    """Pure: returns the next state (the input is not modified).  Stale-term events are ignored."""
    import copy
    s = copy.deepcopy(state)
    if ev.term < s.term:
        return s
    s.term = ev.term
    d = ev.data
    if ev.kind == "member_join":
        s.members[d["node"]] = {"status": "alive", "gpus": d.get("gpus", 0)}
    elif ev.kind == "member_suspect":
        if d["node"] in s.members:
            s.members[d["node"]]["status"] = "suspect"
    elif ev.kind == "member_leave":
        s.members.pop(d["node"], None)
        for inst in s.instances.values():
            if d["node"] in inst["nodes"]:
                inst["status"] = "degraded"
    elif ev.kind == "instance_up":
        s.instances[d["instance"]] = {"model": d["model"], "nodes": list(d["nodes"]), "status": "ready",
                                      "plan_epoch": s.plan_epoch}
    elif ev.kind == "instance_down":
        s.instances.pop(d["instance"], None)
    elif ev.kind == "plan":
        s.plan_epoch += 1
        if d.get("instance") in s.instances:
            s.instances[d["instance"]]["plan_epoch"] = s.plan_epoch
    else:
        raise ValueError(f"unknown event kind {ev.kind!r}")
    s.applied += 1
    return s


class EventLog:
    """Append-only log; entry i carries hash(prev_hash || event)."""

    def __init__(self):
        self.entries: list[tuple[bytes, Event]] = []

    @property
    def head(self) -> bytes:
        return self.entries[-1][0] if self.entries else b"\0" * 32

    def append(self, ev: Event) -> bytes:
        h = hashlib.sha256(self.head + ev.encode()).digest()
        self.entries.append((h, ev))
        return h

    def verify(self) -> bool:
        prev = b"\0" * 32
        for h, ev in self.entries:
            if hashlib.sha256(prev + ev.encode()).digest() != h:
                return False
            prev = h
        return True

    def replay(self) -> ClusterState:
        s = ClusterState()
        for _, ev in self.entries:
            s = apply(s, ev)
        return s
