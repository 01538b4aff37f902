"""Metrics registry backed by the native lock-free Counter/Histogram (csrc/cpu/runtime.cpp),
with a pure-Python fallback, and Prometheus text exposition."""
from __future__ import annotations

import threading


class _PyCounter:
    def __init__(self):
        self.v = 0
        self._l = threading.Lock()

    def add(self, n):
        with self._l:
            self.v += n

    def get(self):
        return self.v


class _PyHist:
    def __init__(self):
        self.vals = []

    def record(self, v):
        self.vals.append(v)

    def quantile(self, q):
        if not self.vals:
            return 0.0
        s = sorted(self.vals)
        return float(s[min(len(s) - 1, int(q * len(s)))])

    def count(self):
        return len(self.vals)

    def sum(self):
        return sum(self.vals)


def _native():
    try:
        from .._ext import ext
        return ext()
    except Exception:
        return None


class Registry:
    def __init__(self, prefix: str = "syntropy_"):
        self.prefix = prefix
        self._c: dict = {}
        self._h: dict = {}
        self._g: dict = {}
        self._l = threading.Lock()

    def counter(self, name: str):
        c = self._c.get(name)
        if c is None:
            with self._l:
                c = self._c.get(name)
                if c is None:
                    n = _native()
                    c = n.Counter() if n else _PyCounter()
                    self._c[name] = c
        return c

    def histogram(self, name: str):
        h = self._h.get(name)
        if h is None:
            with self._l:
                h = self._h.get(name)
                if h is None:
                    n = _native()
                    h = n.Histogram() if n else _PyHist()
                    self._h[name] = h
        return h

    def gauge(self, name: str, value: float):
        self._g[name] = value

    def prometheus(self) -> str:
        out = []
        for n, c in sorted(self._c.items()):
            out.append(f"# TYPE {self.prefix}{n} counter\n{self.prefix}{n} {c.get()}")
        for n, v in sorted(self._g.items()):
            out.append(f"# TYPE {self.prefix}{n} gauge\n{self.prefix}{n} {v}")
        for n, h in sorted(self._h.items()):
            lines = [f"# TYPE {self.prefix}{n} summary"]
            for q in (0.5, 0.9, 0.99):
                lines.append(f'{self.prefix}{n}{{quantile="{q}"}} {h.quantile(q)}')
            lines.append(f"{self.prefix}{n}_sum {h.sum()}")
            lines.append(f"{self.prefix}{n}_count {h.count()}")
            out.append("\n".join(lines))
        return "\n".join(out) + "\n"


METRICS = Registry()
