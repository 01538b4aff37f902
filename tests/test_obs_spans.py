"""Span records in a lossy shared-memory ring (a child process produces, the parent drains;
a full ring drops and counts), and cost-term records of a profiled step."""
import os

from syntropy_b200._ext import ext
from syntropy_b200.obs import trace
from syntropy_b200.obs.spans import SpanRing, step_cost_record


def test_span_ring_across_processes_and_drops():
    cap = 16
    region = ext().ShmRegion(f"/syn-spans-{os.getpid()}", SpanRing.bytes_needed(cap) + 64, True)
    base = (region.address() + 63) // 64 * 64
    ring = SpanRing(cap, base, init=True)
    pid = os.fork()
    if pid == 0:  # producer: 20 spans into a 16-slot ring nobody drains yet
        child = SpanRing(cap, base, init=False)
        trace.SINKS.append(child)
        for i in range(20):
            with trace.span("decode_step", i=i):
                with trace.span("layer"):
                    pass
        os._exit(0 if child.dropped == 40 - cap else 1)
    _, status = os.waitpid(pid, 0)
    assert status == 0  # 40 spans offered, 16 kept, the rest dropped without blocking
    recs = ring.drain(names={__import__("zlib").crc32(b"decode_step"): "decode_step",
                             __import__("zlib").crc32(b"layer"): "layer"})
    assert len(recs) == cap
    layers = [r for r in recs if r["name"] == "layer"]
    steps = {r["span_id"]: r for r in recs if r["name"] == "decode_step"}
    assert layers and all(r["t1_ns"] >= r["t0_ns"] for r in recs)
    assert any(r["parent"] in steps and steps[r["parent"]]["trace_id"] == r["trace_id"] for r in layers)


def test_cost_record_groups_segments():
    segs = [("layer0.attention", 0.1), ("layer0.route", 0.02), ("layer0.gate_up", 0.5), ("layer0.cpu_wait", 3.0),
            ("layer0.moe", 0.01), ("lm_head", 0.3), ("sample", 0.05)]
    rec = step_cost_record(7, segs, {"weights": 1.0, "host_tier": 2.5, "total": 9.9})
    assert rec.measured_ms["host_tier"] == 3.0 and abs(rec.measured_ms["experts"] - 0.53) < 1e-9
    assert abs(rec.total_ms - 3.98) < 1e-9 and rec.predicted_ms == {"weights": 1.0, "host_tier": 2.5}
    assert {r["term"] for r in rec.rows()} >= {"attention", "head", "host_tier", "weights"}
