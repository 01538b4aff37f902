"""Background engine loop for serving: one thread owns the LLMEngine (and the GPU stream);
API handlers submit requests and receive per-token events on asyncio queues.

Reference design: the ingress thread that drives generations and polls them into their
streams (crates/api/src/native.rs:109-157, crates/api/src/pipeline/generation.rs:322).
"""
from __future__ import annotations

import asyncio
import itertools
import queue
import threading
import time
from dataclasses import dataclass, field

from ..obs.metrics import METRICS
from .engine import LLMEngine, SamplingParams


@dataclass
class GenEvent:
    kind: str                 # "started" | "tokens" | "done" | "error"
    tokens: list = field(default_factory=list)
    finish_reason: str | None = None
    error: str | None = None
    usage: dict | None = None
    timings: dict | None = None
    status: int = 500  # "error": 400 for a request the engine rejected, 500 for a failed step
    logprobs: list | None = None  # per emitted token, when the request asked for them: on "tokens"
    #                               the records of that event's tokens, on "done" all of them


class AsyncEngine:
    def __init__(self, engine: LLMEngine):
        self.engine = engine
        self._intake: queue.Queue = queue.Queue()
        self._subs: dict[int, tuple] = {}
        self._wake = threading.Event()
        self._stop = False
        self._thread = threading.Thread(target=self._loop, name="syn-engine", daemon=True)
        self._ids = itertools.count()
        self.ready = False
        self._thread.start()

    def close(self):
        self._stop = True
        self._wake.set()
        self._thread.join(timeout=10)

    # ------------------------------------------------------------------ API side
    async def generate(self, prompt: list[int], params: SamplingParams):
        """Async iterator of GenEvent for one request."""
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        ticket = next(self._ids)
        self._intake.put(("add", ticket, prompt, params, loop, q))
        self._wake.set()
        try:
            while True:
                ev = await q.get()
                yield ev
                if ev.kind in ("done", "error"):
                    return
        finally:
            self._intake.put(("cancel", ticket))
            self._wake.set()

    # ------------------------------------------------------------------ engine thread
    def _emit(self, loop, q, ev):
        loop.call_soon_threadsafe(q.put_nowait, ev)

    def _loop(self):
        eng = self.engine
        ticket_to_seq: dict[int, int] = {}
        self.ready = True
        while not self._stop:
            try:
                while True:
                    msg = self._intake.get_nowait()
                    if msg[0] == "add":
                        _, ticket, prompt, params, loop, q = msg
                        try:
                            sid = eng.add_request(prompt, params)
                        except Exception as e:  # invalid request
                            self._emit(loop, q, GenEvent("error", error=str(e), status=400))
                            continue
                        ticket_to_seq[ticket] = sid
                        self._subs[sid] = (loop, q, time.perf_counter(), len(prompt))
                        self._emit(loop, q, GenEvent("started", usage={"prompt_tokens": len(prompt)}))
                        METRICS.counter("requests_total").add(1)
                    elif msg[0] == "cancel":
                        sid = ticket_to_seq.pop(msg[1], None)
                        if sid is not None and sid in self._subs:
                            eng.abort(sid)
                            self._subs.pop(sid, None)
            except queue.Empty:
                pass
            if not eng.has_work():
                self._wake.wait(timeout=0.05)
                self._wake.clear()
                continue
            t0 = time.perf_counter()
            try:
                outs = eng.step()
            except Exception as e:  # device or internal failure: fail every live request
                for sid, (loop, q, _, _) in list(self._subs.items()):
                    self._emit(loop, q, GenEvent("error", error=f"engine step failed: {e}"))
                    try:  # the failed sequences leave the engine, so later requests are served
                        eng.abort(sid)
                    except Exception:  # noqa: BLE001
                        pass
                self._subs.clear()
                continue
            METRICS.histogram("step_us").record(int((time.perf_counter() - t0) * 1e6))
            _engine_gauges(eng)
            for o in outs:
                sub = self._subs.get(o.seq_id)
                if sub is None:
                    continue
                loop, q, t_arr, n_prompt = sub
                self._emit(loop, q, GenEvent("tokens", tokens=o.new_tokens, logprobs=o.logprobs))
                METRICS.counter("generated_tokens_total").add(len(o.new_tokens))
                if o.finished:
                    s = eng.finished.get(o.seq_id)
                    n_out = len(s.output) if s else 0
                    ttft = (s.t_first_token - s.t_arrival) if s and s.t_first_token else None
                    if ttft is not None:
                        METRICS.histogram("ttft_us").record(int(ttft * 1e6))
                    self._emit(loop, q, GenEvent("done", finish_reason=o.finish_reason,
                                                 usage={"prompt_tokens": n_prompt, "completion_tokens": n_out},
                                                 timings={"ttft_ms": None if ttft is None else ttft * 1e3,
                                                          "total_ms": (time.perf_counter() - t_arr) * 1e3},
                                                 logprobs=(s.logprobs if s and s.params.logprobs is not None
                                                           else None)))
                    self._subs.pop(o.seq_id, None)


def _engine_gauges(eng):
    """Engine state after a step, as gauges: queues, free KV pages, preemption and spill to host
    memory / files, speculative acceptance and the expert cache's VRAM hit rate."""
    st = eng.stats
    METRICS.gauge("running_sequences", len(eng.running))
    METRICS.gauge("waiting_sequences", len(eng.waiting))
    METRICS.gauge("swapped_sequences", len(eng.swapped))
    METRICS.gauge("kv_pages_free", eng.runner.kv.alloc.num_free)
    METRICS.gauge("kv_swapped_out_total", st.get("swapped_out", 0))
    store = getattr(eng, "kv_store", None)
    if store is not None:
        METRICS.gauge("kv_host_swap_bytes", store.host_bytes)
        METRICS.gauge("kv_spill_file_bytes", store.disk_bytes)
    if eng.spec is not None:
        METRICS.gauge("spec_acceptance_rate", round(eng.acceptance_rate, 4))
        METRICS.gauge("spec_paused_steps_total", st.get("spec_paused_steps", 0))
    hr = getattr(eng.runner, "expert_hit_rate", None)
    if hr is not None:
        METRICS.gauge("expert_vram_hit_rate", round(hr, 4))
