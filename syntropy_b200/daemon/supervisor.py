"""Runner supervision as a sans-I/O protocol core driven by explicit time.

The supervisor sees heartbeats and step counters; it declares a runner hung when no
heartbeat arrives for `liveness_timeout_s`, stalled when heartbeats continue but the step
counter does not advance for `stall_factor x predicted step` (and work is pending), and
restarts it with exponential back-off (1 s doubling to 60 s, with jitter) under a restart
budget per window.  Sticky device errors skip the budget and report a device failure.
Reference: crates/daemon/src/supervisor.rs:50-218; RFC-0001 :240-270.
"""
from __future__ import annotations

import enum
import random
from dataclasses import dataclass, field


class RunnerHealth(enum.Enum):
    STARTING = "starting"
    HEALTHY = "healthy"
    HUNG = "hung"
    STALLED = "stalled"
    EXITED = "exited"
    BACKOFF = "backoff"
    FAILED = "failed"


@dataclass
class SupervisorConfig:
    liveness_timeout_s: float = 5.0
    stall_factor: float = 50.0
    min_stall_s: float = 10.0
    backoff_initial_s: float = 1.0
    backoff_max_s: float = 60.0
    jitter: float = 0.1
    restart_budget: int = 5
    budget_window_s: float = 600.0
    seed: int = 0


@dataclass
class Supervisor:
    cfg: SupervisorConfig = field(default_factory=SupervisorConfig)
    state: RunnerHealth = RunnerHealth.STARTING
    last_heartbeat: float = 0.0
    last_step: int = -1
    last_progress: float = 0.0
    predicted_step_s: float = 0.05
    pending_work: bool = False
    restarts: list = field(default_factory=list)
    backoff_s: float = 0.0
    restart_at: float | None = None
    reason: str | None = None

    def __post_init__(self):
        self._rng = random.Random(self.cfg.seed)

    # ---- inputs
    def on_start(self, now: float):
        self.state = RunnerHealth.STARTING
        self.last_heartbeat = now
        self.last_progress = now
        self.restart_at = None

    def on_heartbeat(self, now: float, step: int, pending_work: bool, predicted_step_s: float | None = None):
        self.last_heartbeat = now
        self.pending_work = pending_work
        if predicted_step_s:
            self.predicted_step_s = predicted_step_s
        if step != self.last_step:
            self.last_step = step
            self.last_progress = now
        if self.state in (RunnerHealth.STARTING, RunnerHealth.STALLED):
            self.state = RunnerHealth.HEALTHY

    def on_exit(self, now: float, code: int, device_error: bool = False):
        self.reason = f"exit code {code}" + (" (device error)" if device_error else "")
        if device_error:
            self.state = RunnerHealth.FAILED
            return
        self._schedule_restart(now, RunnerHealth.EXITED)

    # ---- evaluation
    def tick(self, now: float) -> str | None:
        """Returns an action: "kill", "restart", "report_failed" or None."""
        if self.state == RunnerHealth.BACKOFF:
            if self.restart_at is not None and now >= self.restart_at:
                self.on_start(now)
                return "restart"
            return None
        if self.state in (RunnerHealth.FAILED, RunnerHealth.EXITED):
            return "report_failed" if self.state == RunnerHealth.FAILED else None
        if now - self.last_heartbeat > self.cfg.liveness_timeout_s:
            self.reason = "hung: no heartbeat"
            self._schedule_restart(now, RunnerHealth.HUNG)
            return "kill"
        stall = max(self.cfg.min_stall_s, self.cfg.stall_factor * self.predicted_step_s)
        if self.state == RunnerHealth.HEALTHY and self.pending_work and now - self.last_progress > stall:
            self.reason = "stalled: no step progress"
            self._schedule_restart(now, RunnerHealth.STALLED)
            return "kill"
        return None

    def _schedule_restart(self, now: float, why: RunnerHealth):
        self.restarts = [t for t in self.restarts if now - t < self.cfg.budget_window_s]
        if len(self.restarts) >= self.cfg.restart_budget:
            self.state = RunnerHealth.FAILED
            self.reason = (self.reason or why.value) + "; restart budget exhausted"
            return
        self.restarts.append(now)
        n = len(self.restarts)
        base = min(self.cfg.backoff_max_s, self.cfg.backoff_initial_s * (2 ** (n - 1)))
        self.backoff_s = base * (1.0 + self.cfg.jitter * (2 * self._rng.random() - 1))
        self.restart_at = now + self.backoff_s
        self.state = RunnerHealth.BACKOFF
