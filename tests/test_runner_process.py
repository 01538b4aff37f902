"""Runner process model on CPU: the daemon-side RunnerHost spawns a real runner process
(`python -m syntropy_b200 __runner`), completes the Hello / Init handshake over a socket pair,
reads heartbeats and step counters from the shared-memory status header, and the Supervisor
drives kills and restarts with back-off.  Failures are made on the host: the test kills the
CPU runner process by its pid, or stops its heartbeats through a test hook."""
import os
import signal
import time

import pytest
import torch

from syntropy_b200.daemon.runner_host import RunnerHost, RunnerUnavailable
from syntropy_b200.daemon.supervisor import RunnerHealth, SupervisorConfig
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

INIT = {"model": "tiny-llama", "device": "cpu", "seed": 3, "max_batch": 4, "max_seq_len": 128, "heartbeat_ms": 50,
        "test_hooks": True}
PROMPTS = [[5, 6, 7, 8], [100, 200, 300]]


def _want():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, "cpu", seed=3, max_pos=144)
    return LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(PROMPTS, SamplingParams(max_tokens=5))


def _pump(host, until, timeout=60.0):
    t0 = time.monotonic()
    while time.monotonic() - t0 < timeout:
        act = host.poll()
        if until(act):
            return act
        time.sleep(0.02)
    raise AssertionError(f"timed out; events {host.events}")


def _gen(host):
    return host.request({"type": "generate", "prompts": PROMPTS, "params": {"max_tokens": 5}})["outputs"]


def test_spawn_handshake_generate_and_restart_after_kill():
    sup = SupervisorConfig(liveness_timeout_s=2.0, backoff_initial_s=0.05, backoff_max_s=0.2, restart_budget=3)
    host = RunnerHost(INIT, sup)
    host.start()
    try:
        assert host.hello["protocol"] == 1 and host.hello["pid"] == host.pid
        assert host.hdr.state == "ready"
        want = _want()
        assert _gen(host) == want
        assert host.hdr.step > 0  # the step counter moved with the engine
        _pump(host, lambda a: host.sup.state == RunnerHealth.HEALTHY)
        pid = host.pid
        os.kill(pid, signal.SIGKILL)  # a CPU runner process dies
        _pump(host, lambda a: a == "restart")
        assert host.pid is not None and host.pid != pid and host.spawns == 2
        assert _gen(host) == want
    finally:
        host.stop()
    assert any(e.startswith("exit") for _, e in host.events)


def test_hang_is_killed_and_restarted():
    sup = SupervisorConfig(liveness_timeout_s=0.5, backoff_initial_s=0.05, backoff_max_s=0.2, restart_budget=3)
    host = RunnerHost(INIT, sup)
    host.start()
    try:
        _pump(host, lambda a: host.sup.state == RunnerHealth.HEALTHY)
        pid = host.pid
        host.request({"type": "test_stop_heartbeat"})  # the runner stops beating: a hang
        _pump(host, lambda a: a == "kill")
        assert "hung" in host.sup.reason
        _pump(host, lambda a: a == "restart")
        assert host.pid != pid
        assert _gen(host) == _want()
    finally:
        host.stop()


def test_restart_budget_exhausted_reports_failure():
    sup = SupervisorConfig(liveness_timeout_s=5.0, backoff_initial_s=0.01, backoff_max_s=0.02, restart_budget=1)
    host = RunnerHost(INIT, sup)
    host.start()
    try:
        os.kill(host.pid, signal.SIGKILL)
        _pump(host, lambda a: a == "restart")
        os.kill(host.pid, signal.SIGKILL)
        _pump(host, lambda a: a == "failed")
        assert host.sup.state == RunnerHealth.FAILED and "budget" in host.sup.reason
        with pytest.raises(RunnerUnavailable):
            _gen(host)
    finally:
        host.stop()


def test_runner_exits_when_the_daemon_goes_away():
    host = RunnerHost(INIT, SupervisorConfig())
    host.start()
    proc = host.proc
    host.ch.close()  # the daemon's end of the channel closes
    proc.wait(timeout=30)
    assert proc.returncode == 0
    host.proc = None
    host.stop()


def test_ps_lists_the_runner():
    """`ps` reads each runner's shared-memory status header: the spawned runner appears with
    its pid, state and heartbeat; after the daemon side stops it, its region is gone."""
    from syntropy_b200.cli.main import runner_table
    sup = SupervisorConfig(liveness_timeout_s=2.0, backoff_initial_s=0.05, backoff_max_s=0.2, restart_budget=3)
    host = RunnerHost(INIT, sup)
    host.start()
    try:
        _pump(host, lambda a: host.sup.state == RunnerHealth.HEALTHY)
        rows = [r for r in runner_table() if r["pid"] == host.pid]
        assert len(rows) == 1 and rows[0]["state"] == "ready" and rows[0]["alive"]
        assert rows[0]["daemon_pid"] == os.getpid() and rows[0]["heartbeat_age_s"] < 2.0
        region = rows[0]["region"]
    finally:
        host.stop()
    assert all(r["region"] != region for r in runner_table())
