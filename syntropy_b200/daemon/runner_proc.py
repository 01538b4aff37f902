"""The runner process: one per model instance, started by the daemon's RunnerHost.

`serve(fd, region)` is the process body (reached as `python -m syntropy_b200 __runner --ipc-fd
FD --region NAME`):

1. sends `hello` on the inherited channel and waits for `init` (a protocol mismatch or a
   silent daemon ends the process);
2. attaches the shared-memory status region named by the daemon, publishes its pid and
   lifecycle state, and starts the heartbeat thread (every `heartbeat_ms`);
3. Loading -> Warming -> Ready: builds the engine of the model `init` names on its device;
4. serves requests (`generate`, `stats`, `shutdown`) until the daemon says shutdown or goes
   away: a closed channel means the daemon is gone, and the runner exits rather than live on
   as an orphan (the bounded orphan rule).  The step counter advances with every engine step.

Reference: crates/runner/src/process.rs:219 (`serve`: heartbeat thread, daemon watch),
crates/runner/src/lifecycle.rs:38-199.
"""
from __future__ import annotations

import os
import socket
import threading
import time

from ..net.ipc import HEADER_BYTES, PROTOCOL, Channel, ChannelClosed, StatusHeader
from .lifecycle import Lifecycle, LifecycleState


def _build_engine(init: dict):
    import torch

    from ..models.config import get_config
    from ..models.transformer import prepare_weights
    from ..runtime.engine import LLMEngine
    from ..runtime.runner import ModelRunner
    cfg = get_config(init["model"])
    dev = torch.device(init.get("device", "cpu"))
    mw = prepare_weights(cfg, dev, seed=int(init.get("seed", 0)), max_pos=int(init.get("max_seq_len", 256)) + 16)
    runner = ModelRunner(mw, max_batch=int(init.get("max_batch", 4)), max_seq_len=int(init.get("max_seq_len", 256)),
                         use_graphs=dev.type == "cuda")
    return LLMEngine(runner)


def serve(fd: int, region: str) -> int:
    from .._ext import ext
    ch = Channel(socket.socket(fileno=fd))
    life = Lifecycle()
    ch.send({"type": "hello", "protocol": PROTOCOL, "pid": os.getpid(), "build": _build_id()})
    try:
        init = ch.recv(timeout=30.0)
    except ChannelClosed:
        return 2
    if not init or init.get("type") != "init" or init.get("protocol") != PROTOCOL:
        return 2
    shm = ext().ShmRegion(region, int(init.get("region_bytes", HEADER_BYTES)), False)
    hdr = StatusHeader(shm.address())
    hdr.set_pid(os.getpid())  # the header names its runner (read by `ps` and by the daemon)
    stop_beats = threading.Event()
    done = threading.Event()
    period = float(init.get("heartbeat_ms", 100)) / 1e3

    def beats():
        while not done.is_set():
            if not stop_beats.is_set():
                hdr.beat()
            done.wait(period)
    hdr.beat()
    threading.Thread(target=beats, name="syn-heartbeat", daemon=True).start()
    try:
        life.to(LifecycleState.LOADING)
        hdr.set_state("loading")
        eng = _build_engine(init)
        life.to(LifecycleState.WARMING)
        hdr.set_state("warming")
        steps = [0]
        orig_step = eng.step

        def counted_step():
            out = orig_step()
            steps[0] += 1
            hdr.set_step(steps[0])
            return out
        eng.step = counted_step
        life.to(LifecycleState.READY)
        hdr.set_state("ready")
        ch.send({"type": "ready", "durations": life.durations()})
        while True:
            try:
                msg = ch.recv(timeout=0.1)
            except ChannelClosed:
                return 0  # the daemon is gone: no orphan runner
            if msg is None:
                continue
            kind = msg.get("type")
            rid = msg.get("id")
            if kind == "generate":
                from ..runtime.engine import SamplingParams
                hdr.set_pending(True)
                try:
                    sp = SamplingParams(**msg.get("params", {}))
                    out = eng.generate(msg["prompts"], sp)
                    ch.send({"type": "result", "id": rid, "outputs": out})
                except Exception as e:  # noqa: BLE001  (a bad request: reported, the runner lives on)
                    ch.send({"type": "error", "id": rid, "error": f"{type(e).__name__}: {e}"})
                finally:
                    hdr.set_pending(False)
            elif kind == "stats":
                ch.send({"type": "result", "id": rid, "steps": steps[0], "state": life.state.value})
            elif kind == "test_stop_heartbeat" and init.get("test_hooks"):
                stop_beats.set()  # a hang as the supervisor sees it (tests only)
                ch.send({"type": "result", "id": rid})
            elif kind == "shutdown":
                life.to(LifecycleState.DRAINING)
                hdr.set_state("draining")
                life.to(LifecycleState.STOPPED)
                hdr.set_state("stopped")
                ch.send({"type": "result", "id": rid})
                return 0
            else:
                ch.send({"type": "error", "id": rid, "error": f"unknown request {kind!r}"})
    except ChannelClosed:
        return 0
    except Exception as e:  # noqa: BLE001
        life.to(LifecycleState.FAILED, str(e))
        hdr.set_state("failed")
        hdr.set_error(1)
        try:
            ch.send({"type": "failed", "error": f"{type(e).__name__}: {e}"})
        except ChannelClosed:
            pass
        return 1
    finally:
        done.set()
        ch.close()


def _build_id() -> str:
    try:
        from .. import __version__
        return str(getattr(__version__, "__version__", __version__))
    except Exception:  # noqa: BLE001
        return "dev"
