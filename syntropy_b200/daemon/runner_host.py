"""Daemon side of a runner process: spawn, handshake, watch, kill and restart.

`RunnerHost` starts `python -m syntropy_b200 __runner` with one end of a socket pair and the
name of a fresh shared-memory status region, completes the Hello / Init handshake, and then
`poll()` feeds the `Supervisor` protocol core from what it observes: the status header's
heartbeat and step counter, and the process's exit.  The supervisor's decisions are carried
out here: "kill" ends the process (SIGKILL to that exact pid), "restart" spawns a fresh one
after the back-off, "report_failed" leaves the host in the failed state (restart budget
spent, or a device error).  Requests go through `request()`, which fails fast while the
runner is down.

Reference: crates/daemon/src/runner_host.rs:57-666 (`spawn_process` :556), crates/daemon/src/
supervisor.rs:50-218, RFC-0001 :240-270.
"""
from __future__ import annotations

import itertools
import os
import signal
import subprocess
import sys
import time
import uuid

from ..net.ipc import HEADER_BYTES, PROTOCOL, ChannelClosed, StatusHeader, pair
from .supervisor import RunnerHealth, Supervisor, SupervisorConfig


class RunnerUnavailable(RuntimeError):
    """The runner is down (restarting, or failed for good)."""


class RunnerHost:
    def __init__(self, init: dict, sup: SupervisorConfig | None = None, clock=time.monotonic,
                 handshake_timeout_s: float = 120.0, env: dict | None = None):
        self.init = dict(init)
        self.sup = Supervisor(sup or SupervisorConfig())
        self.clock = clock
        self.handshake_timeout_s = handshake_timeout_s
        self.env = env
        self.proc: subprocess.Popen | None = None
        self.ch = None
        self.region = None
        self.hdr: StatusHeader | None = None
        self.hello: dict | None = None
        self.spawns = 0
        self.events: list[tuple[float, str]] = []
        self._ids = itertools.count()

    # ------------------------------------------------------------------ lifecycle
    def start(self):
        """Spawn a runner and complete its handshake (raises if it does not become ready)."""
        from .._ext import ext
        name = f"/syn-runner-{os.getpid()}-{uuid.uuid4().hex[:8]}"
        self.region = ext().ShmRegion(name, HEADER_BYTES, True)
        self.hdr = StatusHeader(self.region.address())
        self.hdr.format(0)
        self.ch, child = pair()
        cmd = [sys.executable, "-m", "syntropy_b200", "__runner", "--ipc-fd", str(child.fileno()), "--region", name]
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env = dict(os.environ if self.env is None else self.env)
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        self.proc = subprocess.Popen(cmd, pass_fds=(child.fileno(),), env=env, stdin=subprocess.DEVNULL)
        child.close()
        self.spawns += 1
        now = self.clock()
        self.sup.on_start(now)
        self._event("spawn", now)
        hello = self.ch.recv(timeout=self.handshake_timeout_s)
        if not hello or hello.get("type") != "hello" or hello.get("protocol") != PROTOCOL:
            self._kill()
            raise RuntimeError(f"runner handshake failed: {hello!r}")
        self.hello = hello
        self.ch.send({"type": "init", "protocol": PROTOCOL, "region": name, "region_bytes": HEADER_BYTES, **self.init})
        ready = self.ch.recv(timeout=self.handshake_timeout_s)
        if not ready or ready.get("type") != "ready":
            self._kill()
            raise RuntimeError(f"runner did not become ready: {ready!r}")
        self._event("ready", self.clock())

    def stop(self):
        if self.proc is not None and self.proc.poll() is None:
            try:
                self.ch.send({"type": "shutdown", "id": next(self._ids)})
                self.ch.recv(timeout=10.0)
            except ChannelClosed:
                pass
            try:
                self.proc.wait(timeout=10.0)
            except subprocess.TimeoutExpired:
                self._kill()
        self._close()
        # the status region goes with the instance (its owner unlinks it): the header view first
        self.hdr = None
        self.region = None

    # ------------------------------------------------------------------ supervision
    def poll(self) -> str | None:
        """One supervision pass; returns the action taken ("kill", "restart", "failed") or None."""
        now = self.clock()
        if self.sup.state == RunnerHealth.FAILED:
            return "failed"
        if self.proc is not None:
            code = self.proc.poll()
            if code is not None:
                self._event(f"exit {code}", now)
                self._close()
                self.sup.on_exit(now, code, device_error=self.hdr_error == 2)
            elif self.hdr is not None and self.hdr.valid():
                hb = self.hdr.heartbeat_ns
                if hb:
                    age = max(0.0, (time.monotonic_ns() - hb) / 1e9)
                    if age <= self.sup.cfg.liveness_timeout_s:
                        self.sup.on_heartbeat(now - age, self.hdr.step, self.hdr.pending)
        act = self.sup.tick(now)
        if act == "kill":
            self._event("kill: " + (self.sup.reason or ""), now)
            self._kill()
            return "kill"
        if act == "restart":
            self._event("restart", now)
            self.start()
            return "restart"
        if act == "report_failed":
            self._event("failed: " + (self.sup.reason or ""), now)
            return "failed"
        return None

    @property
    def hdr_error(self) -> int:
        return self.hdr.error if self.hdr is not None else 0

    @property
    def pid(self) -> int | None:
        return self.proc.pid if self.proc is not None and self.proc.poll() is None else None

    def request(self, msg: dict, timeout: float = 300.0) -> dict:
        if self.proc is None or self.proc.poll() is not None:
            raise RunnerUnavailable(f"runner is {self.sup.state.value}")
        rid = next(self._ids)
        self.ch.send({**msg, "id": rid})
        while True:
            rep = self.ch.recv(timeout=timeout)
            if rep is None:
                raise TimeoutError("runner did not answer")
            if rep.get("id") == rid:
                if rep.get("type") == "error":
                    raise RuntimeError(rep.get("error"))
                return rep

    # ------------------------------------------------------------------ internals
    def _event(self, what: str, t: float):
        self.events.append((t, what))

    def _kill(self):
        if self.proc is not None and self.proc.poll() is None:
            os.kill(self.proc.pid, signal.SIGKILL)
            try:
                self.proc.wait(timeout=10.0)
            except subprocess.TimeoutExpired:
                pass
        self._close()

    def _close(self):
        if self.ch is not None:
            self.ch.close()
            self.ch = None
        self.proc = None
