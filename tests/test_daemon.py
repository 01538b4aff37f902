"""Supervisor protocol on virtual time, lifecycle transitions, fault plans, tracing."""
import pytest

from syntropy_b200.core.errors import SynError
from syntropy_b200.daemon import Lifecycle, LifecycleState, RunnerHealth, Supervisor, SupervisorConfig
from syntropy_b200.obs.faults import FaultPlan, FaultRule, fault_point, install
from syntropy_b200.obs.trace import FLIGHT, parse_traceparent, span, traceparent


def test_supervisor_hang_backoff_and_budget():
    sv = Supervisor(SupervisorConfig(liveness_timeout_s=5, restart_budget=3, jitter=0.0))
    sv.on_start(0.0)
    sv.on_heartbeat(1.0, 1, True)
    assert sv.tick(4.0) is None and sv.state == RunnerHealth.HEALTHY
    assert sv.tick(6.5) == "kill" and sv.state == RunnerHealth.BACKOFF and sv.backoff_s == 1.0
    assert sv.tick(7.0) is None
    assert sv.tick(7.6) == "restart"
    # second and third failures double the back-off, the fourth exhausts the budget
    sv.on_exit(8.0, 1)
    assert sv.backoff_s == 2.0
    sv.tick(10.1)
    sv.on_exit(11.0, 1)
    assert sv.backoff_s == 4.0
    sv.tick(15.1)
    sv.on_exit(16.0, 1)
    assert sv.state == RunnerHealth.FAILED and "budget" in sv.reason


def test_supervisor_stall_detection_and_device_error():
    sv = Supervisor(SupervisorConfig(min_stall_s=2.0, stall_factor=10))
    sv.on_start(0.0)
    sv.on_heartbeat(0.5, 5, True, predicted_step_s=0.05)
    for t in (1.0, 1.5, 2.0):
        sv.on_heartbeat(t, 5, True)
    assert sv.tick(2.4) is None
    sv.on_heartbeat(2.9, 5, True)
    assert sv.tick(3.0) == "kill" and "stalled" in sv.reason
    sv2 = Supervisor()
    sv2.on_start(0.0)
    sv2.on_exit(1.0, 134, device_error=True)
    assert sv2.tick(2.0) == "report_failed"


def test_lifecycle_transitions():
    t = [0.0]
    lc = Lifecycle(clock=lambda: t[0])
    for s in (LifecycleState.LOADING, LifecycleState.WARMING, LifecycleState.READY):
        t[0] += 1.0
        lc.to(s)
    assert lc.ready and lc.durations()["loading"] == 1.0
    with pytest.raises(ValueError):
        lc.to(LifecycleState.LOADING)
    lc.to(LifecycleState.FAILED, "boom")
    assert lc.state == LifecycleState.FAILED and lc.error == "boom"


def test_fault_plan_nth_probability_drop():
    install(FaultPlan([FaultRule("net.tcp.send", effect="drop", nth=2),
                       FaultRule("io.read", effect="error", p=1.0)]))
    try:
        assert fault_point("net.tcp.send") is False
        assert fault_point("net.tcp.send") is True
        assert fault_point("net.tcp.send") is False
        with pytest.raises(SynError):
            fault_point("io.read")
        assert fault_point("unrelated") is False
    finally:
        install(None)
    plan = FaultPlan.from_json('[{"point": "x.*", "effect": "drop", "p": 0.5, "seed": 3}]')
    fired = [plan.check("x.y") for _ in range(200)]
    assert 60 < sum(fired) < 140
    plan2 = FaultPlan.from_json('[{"point": "x.*", "effect": "drop", "p": 0.5, "seed": 3}]')
    assert [plan2.check("x.y") for _ in range(200)] == fired  # deterministic by seed


def test_spans_and_traceparent():
    with span("step", n=1) as outer:
        with span("layer") as inner:
            pass
    assert inner.parent == outer.span_id and inner.trace_id == outer.trace_id
    assert FLIGHT.dump()[-1]["name"] == "step"
    tp = traceparent(outer.trace_id, outer.span_id)
    assert parse_traceparent(tp) == (outer.trace_id, outer.span_id)
    assert parse_traceparent("garbage") is None
