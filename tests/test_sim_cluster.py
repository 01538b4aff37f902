"""Deterministic simulation on virtual time (testkit.sim): membership over lossy, jittery
links with partitions; the coordinator lease under holder crashes and minority partitions
(never two holders at once); the runner supervisor against a scripted runner; the same seed
gives the same trace hash."""
import pytest

from syntropy_b200.cluster.log import Event, EventLog
from syntropy_b200.cluster.membership import Lease, LeaseConfig, Membership, MembershipConfig, Status
from syntropy_b200.daemon.supervisor import RunnerHealth, Supervisor, SupervisorConfig
from syntropy_b200.testkit import LinkModel, SimFabric, SimWorld

NODES = ["a", "b", "c", "d", "e"]


def _membership_world(seed, loss=0.05, jitter=0.02):
    w = SimWorld(seed)
    fab = SimFabric(w, LinkModel(alpha_s=0.001, jitter_s=jitter, loss=loss))
    members = {n: Membership(n, NODES, MembershipConfig()) for n in NODES}
    log = {n: [] for n in NODES}

    def handler(n):
        def on(src, msg):
            for ev in members[n].on_message(w.now, src, msg):
                log[n].append((w.now, *ev))
                w.record(f"{n}:{ev}")
        return on
    for n in NODES:
        fab.add_node(n, handler(n))

    def tick(n):
        out, evs = members[n].tick(w.now)
        for ev in evs:
            log[n].append((w.now, *ev))
            w.record(f"{n}:{ev}")
        for dst, msg in out:
            fab.send(n, dst, msg)
    for i, n in enumerate(NODES):
        w.every(0.1, tick, n, start=0.01 * i, name=f"tick {n}")
    return w, fab, members, log


def test_membership_detects_partition_and_refutes_after_heal():
    w, fab, members, log = _membership_world(seed=1)
    w.run(until=20.0)
    # 5% loss and jitter: nobody is suspected with 1 s heartbeats and a 3 s suspicion window
    assert all(m.status(p) == Status.ALIVE for m in members.values() for p in m.peers)
    fab.partition(["a", "b"], ["c", "d", "e"])
    w.run(until=30.0)
    assert members["c"].status("a") == Status.FAILED and members["a"].status("c") == Status.FAILED
    assert members["c"].status("d") == Status.ALIVE
    t_fail = [t for t, kind, node in log["c"] if kind == "member_leave" and node == "a"]
    assert t_fail and t_fail[0] - 20.0 <= 8.0  # Failed within 8 s of the partition (SC-25)
    t_susp = [t for t, kind, node in log["c"] if kind == "member_suspect" and node == "a"]
    assert t_susp[0] - 20.0 <= 3.0 + 1.0 + 0.1  # three missed heartbeats (+ one period, one tick)
    fab.heal()
    w.run(until=40.0)
    assert all(m.status(p) == Status.ALIVE for m in members.values() for p in m.peers)
    # the events feed the hash-chained cluster log
    el = EventLog()
    for t, kind, node in log["c"]:
        el.append(Event(kind, 1, {"node": node, "gpus": 8}))
    assert el.verify() and el.replay().members["a"]["status"] == "alive"


def test_same_seed_same_trace():
    h = []
    for seed in (3, 3, 4):
        w, fab, _, _ = _membership_world(seed)
        w.after(5.0, fab.partition, ["a"], ["b", "c", "d", "e"])
        w.run(until=15.0)
        h.append(w.trace_hash)
    assert h[0] == h[1] != h[2]


def _lease_world(seed):
    w = SimWorld(seed)
    fab = SimFabric(w, LinkModel(alpha_s=0.002, jitter_s=0.05, loss=0.02))
    cfg = LeaseConfig(lease_s=5.0, renew_s=1.0, margin_s=0.5)
    leases = {n: Lease(n, NODES, cfg) for n in NODES}
    crashed = set()
    held = []  # (node, term, start, end)
    open_ = {}

    def note(n, evs):
        for kind, term in evs:
            w.record(f"{n}:{kind}:{term}")
            if kind == "lease_acquired":
                open_[n] = (term, w.now)
            elif kind == "lease_lost" and n in open_:
                term0, t0 = open_.pop(n)
                held.append((n, term0, t0, w.now))

    def handler(n):
        def on(src, msg):
            if n in crashed:
                return
            out, evs = leases[n].on_message(w.now, src, msg)
            note(n, evs)
            for dst, m in out:
                fab.send(n, dst, m)
        return on
    for n in NODES:
        fab.add_node(n, handler(n))

    def tick(n):
        if n in crashed:
            return
        out, evs = leases[n].tick(w.now)
        note(n, evs)
        for dst, m in out:
            fab.send(n, dst, m)
        # a node without a live lease in view campaigns (deterministic stagger by seed)
        lz = leases[n]
        if not lz.holding and not lz._live_lease(w.now) and w.rng.random() < 0.05:
            for dst, m in lz.campaign(w.now):
                fab.send(n, dst, m)
    for i, n in enumerate(NODES):
        w.every(0.1, tick, n, start=0.013 * i)
    return w, fab, leases, crashed, held, open_


def _no_overlap(held, open_, now):
    spans = held + [(n, t, t0, now) for n, (t, t0) in open_.items()]
    spans.sort(key=lambda s: s[2])
    for (n1, t1, a1, b1), (n2, t2, a2, b2) in zip(spans, spans[1:]):
        assert a2 >= b1 or n1 == n2, (spans,)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_lease_holder_crash_and_minority_partition(seed):
    w, fab, leases, crashed, held, open_ = _lease_world(seed)
    w.run(until=20.0)
    holders = [n for n in NODES if leases[n].holding]
    assert len(holders) == 1
    h1 = holders[0]
    crashed.add(h1)  # the holder stops (its lease runs out everywhere)
    leases[h1].holding = False
    open_.pop(h1, None)
    w.run(until=40.0)
    h2 = [n for n in NODES if leases[n].holding]
    assert len(h2) == 1 and h2[0] != h1 and leases[h2[0]].held_term > 1
    crashed.clear()
    # the holder lands in a minority: it steps down, the majority side elects a new term
    minority = [h2[0], next(n for n in NODES if n != h2[0] and n != h1)]
    fab.partition(minority, [n for n in NODES if n not in minority])
    w.run(until=70.0)
    assert not leases[h2[0]].holding
    h3 = [n for n in NODES if leases[n].holding]
    assert len(h3) == 1 and h3[0] not in minority
    _no_overlap(held, open_, w.now)


def test_supervisor_on_virtual_time():
    """A scripted runner beats every 100 ms, hangs at t = 5 s, and is killed and restarted with
    back-off by the supervisor driven from the simulated clock."""
    w = SimWorld(0)
    sup = Supervisor(SupervisorConfig(liveness_timeout_s=1.0, backoff_initial_s=0.5, restart_budget=3))
    state = {"alive": True, "step": 0, "kills": [], "restarts": []}
    sup.on_start(0.0)

    def runner():
        if state["alive"] and not (5.0 <= w.now < 1e9 and state.get("hung")):
            state["step"] += 1
            sup.on_heartbeat(w.now, state["step"], pending_work=True)
    w.every(0.1, runner)
    w.at(5.0, lambda: state.update(hung=True))

    def daemon():
        act = sup.tick(w.now)
        if act == "kill":
            state["kills"].append(w.now)
            state["alive"] = False
        elif act == "restart":
            state["restarts"].append(w.now)
            state.update(alive=True, hung=False)
        w.record(f"sup:{sup.state.value}")
    w.every(0.05, daemon)
    w.run(until=10.0)
    assert len(state["kills"]) == 1 and 6.0 <= state["kills"][0] <= 6.2
    assert len(state["restarts"]) == 1 and state["restarts"][0] - state["kills"][0] == pytest.approx(0.5, abs=0.1)
    assert sup.state == RunnerHealth.HEALTHY
