"""Network probe: loopback echo run, RTT summary and histogram, silences and the failure
detector replay under LAN / WAN timings, and the report's no-address check."""
import json

from syntropy_b200.net.probe import (LAN, WAN, EchoServer, build_report, check_report, evaluate, histogram, run,
                                     rtt_summary, silences)


def test_loopback_run_reports():
    srv = EchoServer("127.0.0.1", 0)
    try:
        trace = run("127.0.0.1", srv.port, duration_s=0.6, period_s=0.05)
    finally:
        srv.close()
    assert len(trace) == 12 and all(r["rtt_ms"] is not None and 0 <= r["rtt_ms"] < 1000 for r in trace)
    rep = build_report(trace, 0.05)
    assert rep["hop"]["answered"] == 12 and rep["hop"]["lost"] == 0
    assert sum(b["count"] for b in rep["hop"]["histogram"]) == 12
    assert rep["detector"]["lan"] == [] and rep["detector"]["wan"] == []
    text = json.dumps(rep)
    assert check_report(text) == []


def test_summary_and_histogram():
    s = rtt_summary([float(i) for i in range(1, 1001)])
    assert s["p50_ms"] == 500 and s["p99_ms"] == 990 and s["p999_ms"] == 999 and s["max_ms"] == 1000
    assert rtt_summary([]) is None
    h = histogram([1.0, 1.1, 1.9, 2.0, 0.0005])  # ms -> 1000, 1100, 1900, 2000, 1 (clamped) us
    # [512, 1024) splits into 128-us buckets (1000 -> 896); [1024, 2048) into 256-us ones
    assert [(b["lo_us"], b["count"]) for b in h] == [(1, 1), (896, 1), (1024, 1), (1792, 2)]
    for b in h:
        assert b["lo_us"] < b["hi_us"]


def test_detector_replay():
    # echoes arrive at 1, 2, 3 s, then nothing until 8 s (5 s silence), then 9 s ... 38 s (29 s)
    trace = [{"seq": i, "sent_ms": t - 1, "rtt_ms": 1.0, "arrived_ms": t}
             for i, t in enumerate([1000, 2000, 3000, 8000, 9000, 38000])]
    gaps = silences(trace)
    assert (3000, 5000) in gaps and (9000, 29000) in gaps
    lan = evaluate(LAN, gaps)
    assert [(e["at_ms"], e["outcome"]) for e in lan] == [(3000, "suspect"), (9000, "fail")]
    wan = evaluate(WAN, gaps)
    assert [(e["at_ms"], e["outcome"]) for e in wan] == [(9000, "fail")]
    # a lost echo at the end leaves a running silence
    lost = trace + [{"seq": 6, "sent_ms": 50000, "rtt_ms": None, "arrived_ms": None}]
    assert silences(lost)[-1] == (38000, 12000)
    rep = build_report(lost, 1.0)
    assert rep["hop"]["lost"] == 1 and len(rep["stalls"]) == 3


def test_report_check_rejects_addresses():
    base = json.dumps(build_report([], 1.0))
    assert check_report(base) == []
    for addr in ("10.0.0.12", "fe80::1ff:fe23:4567:890a", "00:1a:2b:3c:4d:5e", "::1",
                 "2001:0db8:85a3:0000:0000:8a2e:0370:7334"):
        bad = json.dumps(build_report([], 1.0) | {"note": f"peer {addr}"})
        assert check_report(bad), addr
    assert check_report("{}")  # schema errors
