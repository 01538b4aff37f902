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
