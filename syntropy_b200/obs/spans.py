"""Span records for a lossy shared-memory ring, and per-step cost-term records.

* `SpanRing`: finished spans as fixed 64-byte binary records pushed into a single-producer
  ring (the native SPSC ring, in-process or inside a shared-memory region a daemon drains).
  A full ring drops the record and counts it: a hot thread never blocks on tracing.  Record:
  trace id (16 B), span id (8 B), parent span id (8 B, 0 = root), start and end (u64 ns each),
  name hash (u32, the name itself is kept in a side table), status (u32), 8 reserved bytes.
* `CostRecord`: a profiled decode step's measured segment times grouped into the planner's
  cost terms and set beside the plan's prediction, so a run shows term by term where time
  went against the model (`step_cost_record`).

Reference: crates/obs/src/trace/span.rs (64-byte span records), crates/obs/src/ring.rs and
drain.rs (lossy rings drained by the daemon), crates/obs/src/cost_term.rs (CostTerm keys).
"""
from __future__ import annotations

import struct
import zlib
from dataclasses import dataclass, field

from .._ext import ext

RECORD = struct.Struct("<16s8s8sQQII8x")
assert RECORD.size == 64


class SpanRing:
    def __init__(self, capacity: int = 4096, address: int | None = None, init: bool = True):
        """In-process ring, or a ring at `address` (64-byte aligned, inside a shared-memory
        region; init formats it, otherwise the existing ring is attached)."""
        e = ext()
        self.ring = e.SpscRing(capacity, RECORD.size) if address is None else \
            e.SpscRing(address, capacity, RECORD.size, init)
        self.dropped = 0
        self.names: dict[int, str] = {}

    @staticmethod
    def bytes_needed(capacity: int) -> int:
        return ext().SpscRing.bytes_needed(capacity, RECORD.size)

    def push(self, span, status: int = 0) -> bool:
        h = zlib.crc32(span.name.encode())
        self.names.setdefault(h, span.name)
        rec = RECORD.pack(bytes.fromhex(span.trace_id), bytes.fromhex(span.span_id),
                          bytes.fromhex(span.parent) if span.parent else b"\0" * 8, span.t0_ns, span.t1_ns, h, status)
        ok = self.ring.push(rec)
        if not ok:
            self.dropped += 1
        return ok

    def drain(self, names: dict | None = None) -> list[dict]:
        names = names if names is not None else self.names
        out = []
        while True:
            b = self.ring.pop()
            if b is None:
                return out
            tid, sid, par, t0, t1, h, st = RECORD.unpack(b)
            out.append({"trace_id": tid.hex(), "span_id": sid.hex(),
                        "parent": None if par == b"\0" * 8 else par.hex(), "t0_ns": t0, "t1_ns": t1,
                        "name": names.get(h, f"#{h:08x}"), "status": st})


# measured segment kinds of a profiled decode step -> the planner's cost terms
SEGMENT_TERMS = {
    "attention": "attention", "route": "experts", "dispatch": "collectives", "build": "collectives",
    "gate_up": "experts", "down": "experts", "cpu_wait": "host_tier", "combine": "collectives", "moe": "experts",
    "ffn": "dense", "lm_head": "head", "sample": "head",
}


@dataclass
class CostRecord:
    step: int
    measured_ms: dict = field(default_factory=dict)
    predicted_ms: dict = field(default_factory=dict)

    @property
    def total_ms(self) -> float:
        return sum(self.measured_ms.values())

    def rows(self) -> list[dict]:
        keys = sorted(set(self.measured_ms) | set(self.predicted_ms))
        return [{"term": k, "measured_ms": round(self.measured_ms.get(k, 0.0), 4),
                 "predicted_ms": round(self.predicted_ms[k], 4) if k in self.predicted_ms else None}
                for k in keys]


def step_cost_record(step: int, segments: list[tuple[str, float]], predicted: dict | None = None) -> CostRecord:
    """Groups a profiled step's (label, ms) segments into cost terms.  Predicted terms are the
    planner's (`price_decode`): weights and kv are set against the measured attention, expert
    and dense time they are spent in."""
    rec = CostRecord(step)
    for label, ms in segments:
        term = SEGMENT_TERMS.get(label.split(".")[-1], "other")
        rec.measured_ms[term] = rec.measured_ms.get(term, 0.0) + ms
    if predicted:
        pr = dict(predicted)
        pr.pop("total", None)
        rec.predicted_ms = {k: float(v) for k, v in pr.items()}
    return rec
