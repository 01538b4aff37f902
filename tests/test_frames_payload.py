"""Activation and Token frame codecs: round trips (f32 / bf16 rows, 64-byte row strides),
parts split at row boundaries and joined back, corruption caught by the CRCs, and fixed bytes
for a fixed frame (a golden vector of the layout)."""
import pytest
import torch

from syntropy_b200._ext import ext
from syntropy_b200.net.frames import (FrameError, decode_activation, decode_tokens, encode_activation,
                                      encode_tokens, join_activation, split_activation)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_activation_round_trip(dtype):
    torch.manual_seed(0)
    rows = torch.randn(7, 2 * 300).to(dtype)  # 2 streams x hidden 300: rows padded to 64 bytes
    spans = [(11, 0, 3, 0), (12, 40, 4, 3)]
    buf = encode_activation(rows, spans, kind="prefill", from_stage=1, to_stage=2, step=9, streams=2, kind_arg=5,
                            kind_flags=1)
    assert len(buf) % 64 == 0
    spec, hdr, sp, got = decode_activation(buf)
    assert spec["ftype"] == 1 and spec["step"] == 9
    assert hdr["kind"] == 1 and hdr["hidden"] == 300 and hdr["streams"] == 2 and hdr["n_rows"] == 7
    assert hdr["kind_arg"] == 5 and hdr["kind_flags"] == 1
    assert sp == spans and torch.equal(got, rows)


def test_parts_split_and_join():
    rows = torch.arange(10 * 64, dtype=torch.float32).view(10, 64)
    spans = [(1, 100, 6, 0), (2, 0, 4, 6)]
    parts = split_activation(rows, spans, 4, kind="prefill")
    assert len(parts) == 3
    hdr, got, sp = join_activation(list(reversed(parts)))
    assert torch.equal(got, rows) and sorted(sp) == sorted(spans)
    with pytest.raises(FrameError):
        join_activation(parts[:2])


def test_corruption_is_rejected():
    buf = bytearray(encode_activation(torch.ones(2, 64), [(1, 0, 2, 0)]))
    buf[-1] ^= 1
    with pytest.raises(FrameError) as e:
        decode_activation(bytes(buf))
    assert e.value.code == 4  # payload CRC
    buf = bytearray(encode_tokens([(5, [1, 2, 3], True, "stop")]))
    buf[64] ^= 1  # first extension byte: covered by the header CRC
    with pytest.raises(FrameError) as e:
        decode_tokens(bytes(buf))
    assert e.value.code == 3
    with pytest.raises(FrameError):  # a token frame is not an activation frame
        decode_activation(encode_tokens([(5, [1], False, None)]))


def test_tokens_round_trip():
    entries = [(7, [1, 2, 3], False, None), (8, [], True, "length"), (2 ** 40, [151935], True, "stop")]
    spec, got = decode_tokens(encode_tokens(entries, step=3, chan_seq=12))
    assert spec["ftype"] == 2 and spec["chan_seq"] == 12 and got == entries


def test_golden_token_frame():
    buf = encode_tokens([(1, [2, 3], True, "stop")], step=4)
    assert len(buf) == 64 + 128 + 8
    assert buf[:6] == b"SYNF\x01\x02"
    ext_ = buf[64:192]
    assert ext_[:8] == bytes([1, 0, 0, 0, 2, 0, 0, 0])                      # 1 entry, 2 tokens
    assert ext_[64:80] == bytes([1, 0, 0, 0, 0, 0, 0, 0, 2, 0, 0, 0, 1, 1, 0, 0])  # seq 1, 2 tokens, stop|finished
    assert buf[192:] == bytes([2, 0, 0, 0, 3, 0, 0, 0])
    assert int.from_bytes(buf[56:60], "little") == ext().crc32c(buf[192:])


def test_activation_and_tokens_over_the_tcp_channel():
    import threading

    from syntropy_b200.net.tcp import TcpChannel, TcpListener
    lst = TcpListener()
    got = {}

    def server():
        ch = lst.accept()
        got["a"] = ch.recv_payload()
        got["t"] = ch.recv_payload()
        ch.grant(2)
        ch.close()
    th = threading.Thread(target=server)
    th.start()
    ch = TcpChannel.connect("127.0.0.1", lst.port)
    rows = torch.randn(3, 128).to(torch.bfloat16)
    ch.send_activation(rows, [(9, 17, 3, 0)], kind="decode", step=4)
    ch.send_tokens([(9, [42], False, None)], step=4)
    th.join(timeout=30)
    ch.close()
    lst.close()
    kind, (spec, hdr, spans, r) = got["a"]
    assert kind == "activation" and spec["chan_seq"] == 1 and torch.equal(r, rows) and spans == [(9, 17, 3, 0)]
    kind, (spec, entries) = got["t"]
    assert kind == "tokens" and spec["chan_seq"] == 2 and entries == [(9, [42], False, None)]


def test_collective_round_trip_and_member_order_reduction():
    from syntropy_b200.net.frames import decode_collective, encode_collective, reduce_collective
    torch.manual_seed(5)
    parts = [torch.randn(7, 1000) for _ in range(3)]  # 1000 f32 = 4000 bytes: rows padded to 64
    frames = [encode_collective(p, "ffn_allreduce", m, 3, layer=12, epoch=4, step=9) for m, p in enumerate(parts)]
    spec, hdr, rows = decode_collective(frames[1])
    assert hdr == {"phase": "ffn_allreduce", "member": 1, "n_members": 3, "layer": 12, "row_offset": 0, "epoch": 4}
    assert spec["step"] == 9 and torch.equal(rows, parts[1])
    want = (parts[0] + parts[1]) + parts[2]
    assert torch.equal(reduce_collective(frames[::-1]), want)  # arrival order does not matter
    with pytest.raises(FrameError):
        reduce_collective(frames[:2])  # a member missing
    bf = encode_collective(parts[0].bfloat16(), "exit_gather", 0, 1, layer=0, row_offset=14)
    _, h, r = decode_collective(bf)
    assert r.dtype == torch.bfloat16 and h["row_offset"] == 14 and torch.equal(r, parts[0].bfloat16())


def test_ep_dispatch_and_combine_round_trip():
    from syntropy_b200.net.frames import (decode_ep_combine, decode_ep_dispatch, encode_ep_combine,
                                          encode_ep_dispatch)
    torch.manual_seed(6)
    rows = torch.randn(5, 256).bfloat16()
    routes = [(3, [(17, 0.25), (2, 0.5)]), (4, [(9, 1.0)]), (10, [(1, 0.125), (5, 0.25), (6, 0.0625)]),
              (11, [(0, 0.75)]), (12, [(31, 0.5), (30, 0.5)])]
    buf = encode_ep_dispatch(rows, routes, src_rank=1, dst_rank=3, layer=40, top_k=8, epoch=2)
    spec, hdr, got_routes, got = decode_ep_dispatch(buf)
    assert hdr == {"src_rank": 1, "dst_rank": 3, "layer": 40, "epoch": 2, "top_k": 8}
    assert got_routes == [(r, [(e, w) for e, w in rt]) for r, rt in routes] and torch.equal(got, rows)
    out = torch.randn(5, 256)
    cb = encode_ep_combine(out, [r for r, _ in routes], src_rank=3, dst_rank=1, layer=40)
    _, h2, ids, rows2 = decode_ep_combine(cb)
    assert ids == [3, 4, 10, 11, 12] and h2["src_rank"] == 3 and torch.equal(rows2, out)
    # more routes than top_k, or a damaged payload, are refused
    with pytest.raises(RuntimeError):
        encode_ep_dispatch(rows[:1], [(0, [(i, 0.1) for i in range(3)])], 0, 1, 0, top_k=2)
    bad = bytearray(buf)
    bad[-5] ^= 0xFF
    with pytest.raises(FrameError):
        decode_ep_dispatch(bytes(bad))
    with pytest.raises(FrameError):
        decode_ep_combine(buf)  # a dispatch frame is not a combine frame


def test_collective_and_ep_frames_over_the_tcp_channel():
    import threading

    from syntropy_b200.net.tcp import TcpChannel, TcpListener
    lst = TcpListener()
    got = []

    def server():
        ch = lst.accept()
        for _ in range(3):
            got.append(ch.recv_payload())
        ch.close()
    th = threading.Thread(target=server)
    th.start()
    ch = TcpChannel.connect("127.0.0.1", lst.port)
    part = torch.randn(2, 64)
    ch.send_collective(part, "attn_allreduce", member=1, n_members=2, layer=3, step=5)
    rows = torch.randn(2, 64).to(torch.bfloat16)
    ch.send_ep_dispatch(rows, [(0, [(4, 0.5)]), (1, [(7, 0.25), (4, 0.75)])], src_rank=0, dst_rank=1, layer=3,
                        top_k=8, step=5)
    ch.send_ep_combine(part, [0, 1], src_rank=1, dst_rank=0, layer=3, step=5)
    th.join(timeout=30)
    ch.close()
    lst.close()
    (k0, (s0, h0, r0)), (k1, (s1, h1, rt1, r1)), (k2, (s2, h2, ids2, r2)) = got
    assert (k0, k1, k2) == ("collective", "ep_dispatch", "ep_combine")
    assert [s["chan_seq"] for s in (s0, s1, s2)] == [1, 2, 3]
    assert h0["phase"] == "attn_allreduce" and torch.equal(r0, part)
    assert rt1 == [(0, [(4, 0.5)]), (1, [(7, 0.25), (4, 0.75)])] and torch.equal(r1, rows)
    assert ids2 == [0, 1] and torch.equal(r2, part)
