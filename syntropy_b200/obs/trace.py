"""Spans, W3C traceparent propagation and a bounded flight recorder (the last N spans kept
in memory for post-mortems).  Reference: crates/obs/src/trace/{span.rs,flight.rs,context.rs}."""
from __future__ import annotations

import os
import threading
import time
from collections import deque
from contextlib import contextmanager
from dataclasses import dataclass


@dataclass
class Span:
    trace_id: str
    span_id: str
    parent: str | None
    name: str
    t0_ns: int
    t1_ns: int = 0
    attrs: dict | None = None


class FlightRecorder:
    def __init__(self, capacity: int = 4096):
        self.buf: deque = deque(maxlen=capacity)
        self._l = threading.Lock()

    def record(self, s: Span):
        with self._l:
            self.buf.append(s)

    def dump(self) -> list[dict]:
        with self._l:
            return [s.__dict__.copy() for s in self.buf]


FLIGHT = FlightRecorder()
SINKS: list = []  # extra span sinks (e.g. obs.spans.SpanRing instances a daemon drains)
_local = threading.local()


def new_id(n: int) -> str:
    return os.urandom(n).hex()


def parse_traceparent(h: str | None) -> tuple[str, str] | None:
    if not h:
        return None
    parts = h.split("-")
    if len(parts) != 4 or len(parts[1]) != 32 or len(parts[2]) != 16:
        return None
    return parts[1], parts[2]


def traceparent(trace_id: str, span_id: str, sampled: bool = True) -> str:
    return f"00-{trace_id}-{span_id}-{'01' if sampled else '00'}"


@contextmanager
def span(name: str, **attrs):
    parent = getattr(_local, "cur", None)
    tid = parent.trace_id if parent else new_id(16)
    s = Span(tid, new_id(8), parent.span_id if parent else None, name, time.monotonic_ns(), attrs=attrs or None)
    _local.cur = s
    try:
        yield s
    finally:
        s.t1_ns = time.monotonic_ns()
        _local.cur = parent
        FLIGHT.record(s)
        for sink in SINKS:
            sink.push(s)
