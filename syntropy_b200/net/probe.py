"""Field network probe: echo round trips between two machines over the framed TCP channel, and
a report of what the membership failure detector would have done with the silences seen.

One side listens (`listen`), the other sends an echo request every `period_s` for `duration_s`
(`run`) and builds a report (`build_report`):

* the hop's RTT summary (p50 / p99 / p99.9 / max) and a log-linear histogram (4 buckets per
  power of two, in microseconds);
* the silences: gaps between two echoes that arrive; those above two periods go to the stall
  log;
* the detector replay (`evaluate`): a two-member cluster raises `Suspect` once its peer has been
  silent for `suspect_after_ms` and fails it at `fail_after_ms`; LAN timings are a 1 s period,
  Suspect after 3 s, fail after 7 s; WAN timings a 2 s period, 8 s and 28 s;
* the trace of every request (sequence, send time, RTT or none when lost), for replay.

The report holds no address: `check_report` rejects text that contains an IPv4, IPv6 or MAC
address.  Reference: crates/netprobe/src/{lib.rs:1-31, detector.rs:1-60, stats.rs:19-62,
report.rs:107-479}.
"""
from __future__ import annotations

import json
import math
import re
import struct
import threading
import time
from dataclasses import dataclass

from .tcp import FrameType, TcpChannel, TcpListener

SCHEMA = 1


@dataclass(frozen=True)
class Timing:
    period_ms: int
    suspect_after_ms: int
    fail_after_ms: int


LAN = Timing(1_000, 3_000, 7_000)
WAN = Timing(2_000, 8_000, 28_000)


# ---------------------------------------------------------------------- endpoints
class EchoServer:
    """Answers every PING frame with the same payload, one thread per connection."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0):
        self.listener = TcpListener(host, port)
        self.port = self.listener.port
        self._stop = threading.Event()
        self._threads = []
        self._accept = threading.Thread(target=self._loop, daemon=True)
        self._accept.start()

    def _loop(self):
        while not self._stop.is_set():
            try:
                ch = self.listener.accept()
            except OSError:
                return
            t = threading.Thread(target=self._serve, args=(ch,), daemon=True)
            t.start()
            self._threads.append(t)

    @staticmethod
    def _serve(ch: TcpChannel):
        try:
            while True:
                ft, _, _, payload = ch.recv()
                if ft == FrameType.CLOSE:
                    break
                if ft == FrameType.PING:
                    ch._write(FrameType.PING, payload)
        except (ConnectionError, OSError, ValueError):
            pass
        finally:
            try:
                ch.sock.close()
            except OSError:
                pass

    def close(self):
        self._stop.set()
        self.listener.close()


def run(host: str, port: int, duration_s: float, period_s: float = 1.0, grace_s: float = 2.0) -> list[dict]:
    """Echo requests every `period_s` for `duration_s`; returns the trace: one record per request
    with `seq`, `sent_ms` (from the start) and `rtt_ms` (None when no echo came back by the end
    plus `grace_s`) and `arrived_ms`."""
    ch = TcpChannel.connect(host, port)
    ch.sock.settimeout(30.0)  # warm-up echo: codec loaded and the peer answering, within a bound
    ch._write(FrameType.PING, struct.pack("<QQ", 2 ** 64 - 1, 0))
    while ch.recv()[0] != FrameType.PING:
        pass
    ch.sock.settimeout(None)
    t0 = time.monotonic_ns()
    sent: dict[int, int] = {}
    trace: dict[int, dict] = {}
    done = threading.Event()

    def receiver():
        try:
            while not done.is_set():
                ft, _, _, payload = ch.recv()
                if ft != FrameType.PING:
                    continue
                now = time.monotonic_ns()
                seq, ts = struct.unpack("<QQ", payload[:16])
                if seq in sent and trace[seq]["rtt_ms"] is None:
                    trace[seq]["rtt_ms"] = (now - ts) / 1e6
                    trace[seq]["arrived_ms"] = (now - t0) / 1e6
        except (ConnectionError, OSError, ValueError):
            pass

    rx = threading.Thread(target=receiver, daemon=True)
    rx.start()
    n = max(1, int(round(duration_s / period_s)))
    for seq in range(n):
        target = t0 + int(seq * period_s * 1e9)
        delay = (target - time.monotonic_ns()) / 1e9
        if delay > 0:
            time.sleep(delay)
        ts = time.monotonic_ns()
        sent[seq] = ts
        trace[seq] = {"seq": seq, "sent_ms": (ts - t0) / 1e6, "rtt_ms": None, "arrived_ms": None}
        try:
            ch._write(FrameType.PING, struct.pack("<QQ", seq, ts))
        except OSError:
            break
    deadline = time.monotonic() + grace_s
    while time.monotonic() < deadline and any(r["rtt_ms"] is None for r in trace.values()):
        time.sleep(0.01)
    done.set()
    ch.close()
    return [trace[s] for s in sorted(trace)]


# ---------------------------------------------------------------------- analysis
def rtt_summary(samples: list[float]) -> dict | None:
    """p50 / p99 / p99.9 / max of RTT samples in ms (nearest rank), None without samples."""
    if not samples:
        return None
    s = sorted(samples)

    def rank(q):
        return s[min(len(s) - 1, max(0, math.ceil(q * len(s)) - 1))]
    return {"count": len(s), "p50_ms": rank(0.5), "p99_ms": rank(0.99), "p999_ms": rank(0.999), "max_ms": s[-1]}


def histogram(samples: list[float]) -> list[dict]:
    """Log-linear buckets over microseconds: each power of two split into 4 equal buckets;
    returns the non-empty ones as {lo_us, hi_us, count}."""
    counts: dict[tuple[int, int], int] = {}
    for ms in samples:
        us = max(1.0, ms * 1e3)
        e = int(math.floor(math.log2(us)))
        sub = min(3, int((us / 2 ** e - 1.0) * 4))
        counts[(e, sub)] = counts.get((e, sub), 0) + 1
    out = []
    for (e, sub), c in sorted(counts.items()):
        lo = 2 ** e * (1 + sub / 4)
        out.append({"lo_us": round(lo, 3), "hi_us": round(lo + 2 ** e / 4, 3), "count": c})
    return out


def silences(trace: list[dict]) -> list[tuple[float, float]]:
    """(start_ms, gap_ms) between consecutive echo arrivals, and from the start to the first."""
    arr = sorted(r["arrived_ms"] for r in trace if r.get("arrived_ms") is not None)
    out, prev = [], 0.0
    for a in arr:
        out.append((prev, a - prev))
        prev = a
    if trace:
        end = max(r["sent_ms"] for r in trace)
        if end > prev:
            out.append((prev, end - prev))  # silence running at the end of the run
    return out


def evaluate(timing: Timing, gaps: list[tuple[float, float]]) -> list[dict]:
    """What the two-member failure detector would have raised for each silence."""
    return [{"at_ms": round(at, 3), "silence_ms": round(g, 3),
             "outcome": "fail" if g >= timing.fail_after_ms else "suspect"}
            for at, g in gaps if g >= timing.suspect_after_ms]


def build_report(trace: list[dict], period_s: float) -> dict:
    rtts = [r["rtt_ms"] for r in trace if r["rtt_ms"] is not None]
    gaps = silences(trace)
    stall_ms = 2 * period_s * 1e3
    return {
        "schema": SCHEMA,
        "settings": {"period_ms": period_s * 1e3, "requests": len(trace)},
        "hop": {"answered": len(rtts), "lost": len(trace) - len(rtts), "rtt": rtt_summary(rtts),
                "histogram": histogram(rtts)},
        "stalls": [{"at_ms": round(a, 3), "silence_ms": round(g, 3)} for a, g in gaps if g > stall_ms],
        "detector": {"lan": evaluate(LAN, gaps), "wan": evaluate(WAN, gaps),
                     "timings": {"lan": LAN.__dict__, "wan": WAN.__dict__}},
        "trace": trace,
    }


_ADDRESS = [
    ("IPv4 address", re.compile(r"(?<![\d.])(?:\d{1,3}\.){3}\d{1,3}(?![\d.])")),
    ("MAC address", re.compile(r"(?i)(?<![0-9a-f:])(?:[0-9a-f]{2}[:-]){5}[0-9a-f]{2}(?![0-9a-f:])")),
    # full form (8 groups) or any run of hex groups and colons that holds "::"
    ("IPv6 address", re.compile(r"(?i)(?<![0-9a-f:])(?=[0-9a-f:]*::|(?:[0-9a-f]{1,4}:){7}[0-9a-f]{1,4})"
                                r"[0-9a-f]{0,4}(?::[0-9a-f]{0,4}){2,7}(?![0-9a-f:])")),
]


def check_report(text: str) -> list[str]:
    """Problems of a report's text: addresses it must not hold, and schema errors."""
    problems = [f"report holds an {name}: {m.group(0)!r}" for name, rx in _ADDRESS for m in rx.finditer(text)]
    try:
        r = json.loads(text)
    except json.JSONDecodeError as e:
        return problems + [f"not JSON: {e}"]
    if r.get("schema") != SCHEMA:
        problems.append(f"schema {r.get('schema')!r}, expected {SCHEMA}")
    for key in ("settings", "hop", "stalls", "detector", "trace"):
        if key not in r:
            problems.append(f"missing {key}")
    return problems


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(prog="syntropy_b200 netprobe")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("listen")
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--port", type=int, default=47000)
    p = sub.add_parser("run")
    p.add_argument("target", help="host:port of the listening side")
    p.add_argument("--duration", type=float, default=60.0, help="seconds")
    p.add_argument("--period", type=float, default=1.0, help="seconds between echo requests")
    p.add_argument("--out", default=None)
    p = sub.add_parser("check")
    p.add_argument("file")
    a = ap.parse_args(argv)
    if a.cmd == "listen":
        srv = EchoServer(a.host, a.port)
        print(f"listening on port {srv.port}; on the other machine run: netprobe run <this-host>:{srv.port}")
        try:
            while True:
                time.sleep(3600)
        except KeyboardInterrupt:
            srv.close()
        return 0
    if a.cmd == "run":
        host, port = a.target.rsplit(":", 1)
        rep = build_report(run(host, int(port), a.duration, a.period), a.period)
        text = json.dumps(rep, indent=1)
        bad = check_report(text)
        if bad:
            raise SystemExit("; ".join(bad))
        out = a.out or f"netprobe-{int(time.time())}.json"
        with open(out, "w") as f:
            f.write(text)
        print(json.dumps({k: rep[k] for k in ("hop", "stalls")} | {"detector": {k: rep["detector"][k]
                                                                              for k in ("lan", "wan")}}))
        print(f"report: {out}")
        return 0
    with open(a.file) as f:
        bad = check_report(f.read())
    print("ok" if not bad else "\n".join(bad))
    return 0 if not bad else 1
