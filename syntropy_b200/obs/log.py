"""Logging pipeline with repeat suppression: an identical (logger, level, message) repeated
within a window is dropped after its first occurrence and summarised once ("... repeated N
times") when it stops or the window ends, so a hot loop that logs cannot flood the sinks.
Reference: crates/daemon/src/logging/* (pipeline, suppression, sinks)."""
from __future__ import annotations

import logging
import threading
import time


class RepeatSuppressor(logging.Filter):
    """Passes the first record of a run of identical records; counts the rest, and reports the
    count with the next different record of the same logger (or on `flush`)."""

    def __init__(self, window_s: float = 5.0):
        super().__init__()
        self.window_s = window_s
        self._last: dict = {}  # logger -> [key, first time, suppressed count, level]
        self._l = threading.Lock()

    def filter(self, record: logging.LogRecord) -> bool:
        key = (record.levelno, record.getMessage())
        now = time.monotonic()
        with self._l:
            st = self._last.get(record.name)
            if st is not None and st[0] == key and now - st[1] < self.window_s:
                st[2] += 1
                return False
            if st is not None and st[2]:
                record.msg = f"{record.msg} (previous message repeated {st[2]} times)"
            self._last[record.name] = [key, now, 0, record.levelno]
        return True

    def flush(self) -> dict:
        """Suppressed counts still pending, per logger (and resets them)."""
        with self._l:
            out = {n: st[2] for n, st in self._last.items() if st[2]}
            for st in self._last.values():
                st[2] = 0
        return out


def install(logger: logging.Logger | None = None, window_s: float = 5.0) -> RepeatSuppressor:
    """Attach a suppressor to every handler of `logger` (the root logger by default)."""
    lg = logger or logging.getLogger()
    f = RepeatSuppressor(window_s)
    for h in lg.handlers or []:
        h.addFilter(f)
    lg.addFilter(f)
    return f
