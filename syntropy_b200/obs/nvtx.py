"""NVTX ranges around the engine's device work, for timelines in Nsight Systems.

Off by default: with SYN_NVTX=1 in the environment (read once, at import), the decorated
calls (the runner's prefill and decode steps) push a named range before and pop it after, so a
timeline shows which kernels belong to which step.  Without it the decorator returns the
function unchanged (no cost on the hot path).  Ranges mark host-side enqueue spans; the kernels
they launch appear under them on the timeline.
"""
from __future__ import annotations

import functools
import os

ENABLED = os.environ.get("SYN_NVTX", "0") == "1"


def nvtx_ranged(name: str):
    def wrap(fn):
        if not ENABLED:
            return fn
        import torch

        @functools.wraps(fn)
        def inner(*a, **k):
            if not torch.cuda.is_available():
                return fn(*a, **k)
            torch.cuda.nvtx.range_push(name)
            try:
                return fn(*a, **k)
            finally:
                torch.cuda.nvtx.range_pop()
        return inner
    return wrap
