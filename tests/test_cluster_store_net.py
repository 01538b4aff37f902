"""Cluster event log (hash chain, pure apply), local model store digests, framed TCP
transport with credits and sequence checks (incl. an injected drop)."""
import threading

import pytest

from syntropy_b200.cluster import ClusterState, Event, EventLog, apply
from syntropy_b200.net import FrameType, TcpChannel, TcpListener
from syntropy_b200.obs.faults import FaultPlan, FaultRule, install
from syntropy_b200.store import ModelStore


def test_event_log_chain_and_apply():
    log = EventLog()
    for ev in (Event("member_join", 1, {"node": "a", "gpus": 8}), Event("member_join", 1, {"node": "b", "gpus": 8}),
               Event("instance_up", 1, {"instance": "i0", "model": "qwen", "nodes": ["a", "b"]}),
               Event("plan", 1, {"instance": "i0"}), Event("member_leave", 2, {"node": "b"}),
               Event("member_join", 1, {"node": "stale"})):
        log.append(ev)
    assert log.verify()
    s = log.replay()
    assert set(s.members) == {"a"} and s.instances["i0"]["status"] == "degraded"
    assert s.instances["i0"]["plan_epoch"] == 1 and s.term == 2
    s0 = ClusterState()
    s1 = apply(s0, Event("member_join", 1, {"node": "x"}))
    assert s0.members == {} and "x" in s1.members  # pure
    log.entries[1] = (log.entries[1][0], Event("member_join", 1, {"node": "evil"}))
    assert not log.verify()


def test_model_store(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    (src / "model.safetensors").write_bytes(b"x" * 1000)
    (src / "config.json").write_text("{}")
    st = ModelStore(str(tmp_path / "store"))
    e = st.add("tiny", str(src))
    assert st.list() == ["tiny"] and len(e["files"]) == 2
    assert st.verify("tiny") == []
    (tmp_path / "store" / "tiny" / "config.json").write_text('{"x":1}')
    assert st.verify("tiny") == ["config.json"]
    assert ModelStore(str(tmp_path / "store")).list() == ["tiny"]


def test_tcp_channel_credits_and_sequence():
    lst = TcpListener()
    got = []

    def server():
        ch = lst.accept(window=4)
        for _ in range(10):
            ft, spec, x, p = ch.recv()
            got.append((ft, spec["chan_seq"], p))
            ch.grant(1)
        ch.close()

    th = threading.Thread(target=server)
    th.start()
    c = TcpChannel.connect("127.0.0.1", lst.port, window=4)
    recv_thread = threading.Thread(target=lambda: _drain_credits(c))
    recv_thread.daemon = True
    recv_thread.start()
    for i in range(10):
        c.send(FrameType.ACTIVATION, bytes([i]) * 100, step=i)
    th.join(timeout=30)
    assert [g[1] for g in got] == list(range(1, 11))
    assert got[3][2] == bytes([3]) * 100
    lst.close()


def _drain_credits(ch):
    try:
        while True:
            ch.recv()
    except Exception:
        pass


def test_tcp_sequence_gap_detected_on_drop():
    lst = TcpListener()
    err = []

    def server():
        ch = lst.accept()
        try:
            for _ in range(3):
                ch.recv()
        except ValueError as e:
            err.append(str(e))

    th = threading.Thread(target=server)
    th.start()
    c = TcpChannel.connect("127.0.0.1", lst.port)
    install(FaultPlan([FaultRule("net.tcp.send", effect="drop", nth=2)]))
    try:
        for i in range(3):
            c.send(FrameType.TOKEN, b"t")
    finally:
        install(None)
    th.join(timeout=30)
    assert err and "sequence gap" in err[0]
    lst.close()
