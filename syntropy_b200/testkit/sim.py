"""Deterministic simulation on virtual time: the multi-node and supervisor logic runs here
without a cluster, a network or real sleeps.

* `SimWorld`: a single-threaded event loop over a virtual clock, with a seeded random source;
  events at equal times run in scheduling order, so one seed gives one history.  Every event
  is folded into a running BLAKE3 digest (`trace_hash`), which tests compare across runs.
* `SimFabric`: message links between named nodes, each with latency (alpha), bandwidth (beta,
  bytes per second), jitter and loss probability; partitions cut sets of links and `heal`
  restores them.  A message in flight when its link is cut is lost.

Reference: crates/testkit/src/sim/world.rs:238 (`SimWorld`), crates/testkit/src/sim/fabric.rs
:254 (`SimFabric`: alpha, beta, jitter, loss, splits), crates/testkit/src/sim/scenario.rs.
"""
from __future__ import annotations

import heapq
import random
import struct
from dataclasses import dataclass


class SimWorld:
    def __init__(self, seed: int = 0):
        self.now = 0.0
        self.rng = random.Random(seed)
        self._q: list = []
        self._n = 0
        self._digest = b"\x00" * 32
        self.events_run = 0

    def at(self, t: float, fn, *args, name: str = ""):
        """Run fn(*args) at virtual time t (>= now)."""
        heapq.heappush(self._q, (max(t, self.now), self._n, fn, args, name or getattr(fn, "__name__", "event")))
        self._n += 1

    def after(self, dt: float, fn, *args, name: str = ""):
        self.at(self.now + dt, fn, *args, name=name)

    def every(self, period: float, fn, *args, name: str = "", start: float | None = None):
        """Run fn(*args) every `period` until it returns False."""
        def tick():
            if fn(*args) is not False:
                self.after(period, tick, name=name)
        self.at(self.now if start is None else start, tick, name=name)

    def run(self, until: float | None = None, max_events: int = 1_000_000):
        while self._q and self.events_run < max_events:
            t, _, fn, args, name = self._q[0]
            if until is not None and t > until:
                break
            heapq.heappop(self._q)
            self.now = t
            self.events_run += 1
            self._fold(name)
            fn(*args)
        if until is not None and self.now < until:
            self.now = until

    def _fold(self, name: str):
        from .._ext import ext
        self._digest = ext().blake3(self._digest + struct.pack("<d", self.now) + name.encode())

    def record(self, what: str):
        """Fold an observation (a state change) into the trace."""
        self._fold("obs:" + what)

    @property
    def trace_hash(self) -> str:
        return self._digest.hex()


@dataclass
class LinkModel:
    alpha_s: float = 0.0005       # one-way latency
    beta_bps: float = 12.5e9      # bytes per second
    jitter_s: float = 0.0         # uniform extra latency in [0, jitter)
    loss: float = 0.0             # drop probability per message


class SimFabric:
    def __init__(self, world: SimWorld, default: LinkModel | None = None):
        self.world = world
        self.default = default or LinkModel()
        self.links: dict[tuple[str, str], LinkModel] = {}
        self.cut: set[frozenset] = set()
        self.handlers: dict[str, object] = {}
        self.delivered = 0
        self.dropped = 0
        self._epoch: dict[frozenset, int] = {}

    def add_node(self, name: str, handler):
        """handler(src, msg) is called on delivery."""
        self.handlers[name] = handler

    def link(self, a: str, b: str) -> LinkModel:
        return self.links.get((a, b)) or self.links.get((b, a)) or self.default

    def set_link(self, a: str, b: str, model: LinkModel):
        self.links[(a, b)] = model

    def partition(self, *groups):
        """Cut every link between different groups (a node in no group keeps all its links)."""
        for i, ga in enumerate(groups):
            for gb in groups[i + 1:]:
                for a in ga:
                    for b in gb:
                        key = frozenset((a, b))
                        self.cut.add(key)
                        self._epoch[key] = self._epoch.get(key, 0) + 1
        self.world.record(f"partition {sorted(map(sorted, groups))}")

    def heal(self):
        self.cut.clear()
        self.world.record("heal")

    def send(self, src: str, dst: str, msg, nbytes: int = 64):
        key = frozenset((src, dst))
        if key in self.cut:
            self.dropped += 1
            return
        m = self.link(src, dst)
        if m.loss and self.world.rng.random() < m.loss:
            self.dropped += 1
            return
        delay = m.alpha_s + nbytes / m.beta_bps + (self.world.rng.random() * m.jitter_s if m.jitter_s else 0.0)
        epoch = self._epoch.get(key, 0)

        def deliver():
            if key in self.cut or self._epoch.get(key, 0) != epoch:
                self.dropped += 1  # the link was cut while the message was in flight
                return
            self.delivered += 1
            h = self.handlers.get(dst)
            if h is not None:
                h(src, msg)
        self.world.after(delay, deliver, name=f"deliver {src}->{dst}")
