"""Framed TCP channel: frames are encoded/verified by the native codec; data frames carry a
channel sequence number (from 1) checked for continuity; the receiver grants credits so a
sender never has more than `window` unacknowledged data frames in flight."""
from __future__ import annotations

import enum
import socket
import struct
import threading

from .._ext import ext
from ..obs.faults import fault_point


class FrameType(enum.IntEnum):
    ACTIVATION = 0x01
    TOKEN = 0x02
    SEQ_CONTROL = 0x03
    CREDIT = 0x04
    KV_CHUNK = 0x05
    COLLECTIVE = 0x08
    STEP_DESCRIPTOR = 0x09
    HELLO = 0x0A
    HELLO_ACK = 0x0B
    CLOSE = 0x0C
    EP_DISPATCH = 0x0E
    EP_COMBINE = 0x0F
    PING = 0x10


CONTROL = {FrameType.HELLO, FrameType.HELLO_ACK, FrameType.CREDIT, FrameType.PING, FrameType.CLOSE}


def _recv_exact(sock, n):
    buf = bytearray()
    while len(buf) < n:
        b = sock.recv(n - len(buf))
        if not b:
            raise ConnectionError("peer closed")
        buf += b
    return bytes(buf)


class TcpChannel:
    def __init__(self, sock: socket.socket, instance: int = 0, window: int = 64):
        self.sock = sock
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self.instance = instance
        self.window = window
        self.send_seq = 0
        self.recv_seq = 0
        self.credits = window
        self._cv = threading.Condition()
        self._lock = threading.Lock()

    @classmethod
    def connect(cls, host: str, port: int, **kw) -> "TcpChannel":
        return cls(socket.create_connection((host, port)), **kw)

    def _write(self, ftype, payload: bytes, ext_b: bytes = b"", step: int = 0, seq: int = 0):
        f = ext().frame_encode(int(ftype), 0, self.instance, 0, 0, step, seq, ext_b, payload)
        with self._lock:
            self.sock.sendall(f)

    def send(self, ftype: FrameType, payload: bytes, ext_b: bytes = b"", step: int = 0, timeout: float = 30.0):
        """Send a data frame; blocks while the receiver has granted no credit."""
        with self._cv:
            if not self._cv.wait_for(lambda: self.credits > 0, timeout=timeout):
                raise TimeoutError("no credit from receiver")
            self.credits -= 1
            self.send_seq += 1
            seq = self.send_seq
        if fault_point("net.tcp.send"):
            return seq  # dropped by a fault plan (the receiver sees a sequence gap)
        self._write(ftype, payload, ext_b, step, seq)
        return seq

    def recv(self):
        """Next data frame as (ftype, spec, ext, payload); credit frames are consumed here."""
        while True:
            hdr = _recv_exact(self.sock, 64)
            ext_len, pay_len = struct.unpack_from("<II", hdr, 48)
            body = _recv_exact(self.sock, ext_len + pay_len)
            self.last_frame = hdr + body
            rc, spec, x, p = ext().frame_decode(self.last_frame)
            if rc != 0:
                raise ValueError(f"bad frame (code {rc})")
            ft = FrameType(spec["ftype"])
            if ft == FrameType.CREDIT:
                with self._cv:
                    self.credits += int.from_bytes(p[:4], "little")
                    self._cv.notify_all()
                continue
            if ft in CONTROL:
                return ft, spec, x, p
            if spec["chan_seq"] != self.recv_seq + 1:
                raise ValueError(f"sequence gap: expected {self.recv_seq + 1}, got {spec['chan_seq']}")
            self.recv_seq = spec["chan_seq"]
            return ft, spec, x, p

    def _send_raw(self, build, timeout: float = 30.0):
        """Send a data frame that `build(chan_seq)` encodes in full (payload codecs)."""
        with self._cv:
            if not self._cv.wait_for(lambda: self.credits > 0, timeout=timeout):
                raise TimeoutError("no credit from receiver")
            self.credits -= 1
            self.send_seq += 1
            seq = self.send_seq
        if fault_point("net.tcp.send"):
            return seq
        f = build(seq)
        with self._lock:
            self.sock.sendall(f)
        return seq

    def send_activation(self, rows, spans, kind: str = "decode", step: int = 0, **kw):
        """Hidden-state rows of a pipeline hand-off as one Activation frame."""
        from .frames import encode_activation
        return self._send_raw(lambda seq: encode_activation(rows, spans, kind=kind, step=step, chan_seq=seq,
                                                            instance=self.instance, **kw))

    def send_tokens(self, entries, step: int = 0):
        """Sampled tokens per sequence as one Token frame."""
        from .frames import encode_tokens
        return self._send_raw(lambda seq: encode_tokens(entries, step=step, chan_seq=seq, instance=self.instance))

    def send_collective(self, rows, phase: str, member: int, n_members: int, layer: int, step: int = 0, **kw):
        """This member's part of a group reduction or gather as one Collective frame."""
        from .frames import encode_collective
        return self._send_raw(lambda seq: encode_collective(rows, phase, member, n_members, layer, step=step,
                                                            chan_seq=seq, instance=self.instance, **kw))

    def send_ep_dispatch(self, rows, routes, src_rank: int, dst_rank: int, layer: int, top_k: int, step: int = 0):
        """Rows for the owner of some of their experts, with their route records."""
        from .frames import encode_ep_dispatch
        return self._send_raw(lambda seq: encode_ep_dispatch(rows, routes, src_rank, dst_rank, layer, top_k,
                                                             step=step, chan_seq=seq, instance=self.instance))

    def send_ep_combine(self, rows, row_ids, src_rank: int, dst_rank: int, layer: int, step: int = 0):
        """The owner's weighted f32 sums, back to the rows' source rank."""
        from .frames import encode_ep_combine
        return self._send_raw(lambda seq: encode_ep_combine(rows, row_ids, src_rank, dst_rank, layer, step=step,
                                                            chan_seq=seq, instance=self.instance))

    def recv_payload(self):
        """Next data frame decoded by its payload codec: ("activation", (spec, header, spans, rows)),
        ("tokens", (spec, entries)), ("collective", (spec, header, rows)), ("ep_dispatch", (spec,
        header, routes, rows)), ("ep_combine", (spec, header, row ids, rows)), or (frame type,
        (spec, ext, payload)) for other types."""
        from . import frames
        ft, spec, x, p = self.recv()
        decoders = {FrameType.ACTIVATION: ("activation", frames.decode_activation),
                    FrameType.TOKEN: ("tokens", frames.decode_tokens),
                    FrameType.COLLECTIVE: ("collective", frames.decode_collective),
                    FrameType.EP_DISPATCH: ("ep_dispatch", frames.decode_ep_dispatch),
                    FrameType.EP_COMBINE: ("ep_combine", frames.decode_ep_combine)}
        if ft in decoders:
            name, dec = decoders[ft]
            return name, dec(self.last_frame)
        return ft, (spec, x, p)

    def grant(self, n: int = 1):
        self._write(FrameType.CREDIT, int(n).to_bytes(4, "little"))

    def close(self):
        try:
            self._write(FrameType.CLOSE, b"")
        except OSError:
            pass
        self.sock.close()


class TcpListener:
    def __init__(self, host: str = "127.0.0.1", port: int = 0):
        self.sock = socket.socket()
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.sock.bind((host, port))
        self.sock.listen(8)
        self.port = self.sock.getsockname()[1]

    def accept(self, **kw) -> TcpChannel:
        s, _ = self.sock.accept()
        return TcpChannel(s, **kw)

    def close(self):
        self.sock.close()
