"""Daemon <-> runner IPC: the command channel and the shared-memory status header.

* `Channel`: length-prefixed msgpack messages over one end of a connected socket pair (the
  runner inherits the other end as a file descriptor).  The runner speaks first with `hello`
  (protocol version, build id, pid); the daemon answers `init` (status-region name, model and
  run settings) or closes the channel on a protocol mismatch.  After that, requests and
  replies carry an `id`.  Reference: crates/ipc/src/cmd.rs:137-473 (channel, Hello / Init
  handshake), crates/ipc/src/cmd/msg.rs:33-192 (messages).
* `StatusHeader`: fixed words at the start of a POSIX shared-memory region (the native
  `ShmRegion`), each on its own 64-byte line so the runner's writes never share a line with the
  daemon's: magic and protocol, runner pid, lifecycle state, heartbeat time (ns, monotonic),
  step counter, pending-work flag, last error code.  The runner's heartbeat thread refreshes
  the heartbeat and the engine loop the step counter; the daemon only reads them (the
  supervisor's liveness and stall inputs).  Reference: crates/ipc/src/shm.rs:75-468 (region,
  header words), RFC-0001 :240-300.
"""
from __future__ import annotations

import ctypes
import select
import socket
import struct
import time

import msgpack

PROTOCOL = 1
MAGIC = 0x53594E52  # "SYNR"
_LEN = struct.Struct("<I")
MAX_MESSAGE = 64 << 20

# status header: one 64-byte line per word group
OFF_MAGIC, OFF_PROTOCOL, OFF_PID, OFF_STATE = 0, 4, 8, 16
OFF_HEARTBEAT = 64     # u64 ns (runner's monotonic clock; CLOCK_MONOTONIC is shared by the host)
OFF_STEP = 128         # u64 engine steps taken
OFF_PENDING = 192      # u32 1 = requests waiting or running
OFF_ERROR = 256        # u32 last error code (0 = none)
HEADER_BYTES = 320

STATES = ["fetching", "packing", "loading", "warming", "ready", "draining", "stopped", "failed"]


class ChannelClosed(Exception):
    """The peer closed its end (or sent a malformed frame)."""


class Channel:
    def __init__(self, sock: socket.socket):
        self.sock = sock
        self._buf = b""

    def send(self, msg: dict):
        data = msgpack.packb(msg, use_bin_type=True)
        if len(data) > MAX_MESSAGE:
            raise ValueError("message too large")
        try:
            self.sock.sendall(_LEN.pack(len(data)) + data)
        except OSError as e:
            raise ChannelClosed(str(e)) from e

    def _fill(self, n: int, deadline: float | None) -> bool:
        while len(self._buf) < n:
            wait = None if deadline is None else max(0.0, deadline - time.monotonic())
            r, _, _ = select.select([self.sock], [], [], wait)
            if not r:
                return False
            try:
                chunk = self.sock.recv(1 << 20)
            except OSError as e:
                raise ChannelClosed(str(e)) from e
            if not chunk:
                raise ChannelClosed("peer closed the channel")
            self._buf += chunk
        return True

    def recv(self, timeout: float | None = None) -> dict | None:
        """The next message, or None if none arrived within `timeout` seconds."""
        deadline = None if timeout is None else time.monotonic() + timeout
        if not self._fill(4, deadline):
            return None
        (n,) = _LEN.unpack(self._buf[:4])
        if n > MAX_MESSAGE:
            raise ChannelClosed("oversized frame")
        if not self._fill(4 + n, None if deadline is None else deadline + 5.0):
            raise ChannelClosed("truncated frame")
        data, self._buf = self._buf[4:4 + n], self._buf[4 + n:]
        msg = msgpack.unpackb(data, raw=False)
        if not isinstance(msg, dict):
            raise ChannelClosed("malformed message")
        return msg

    def close(self):
        try:
            self.sock.close()
        except OSError:
            pass


def pair() -> tuple[Channel, socket.socket]:
    """(daemon-side channel, runner-side socket to hand to the child)."""
    a, b = socket.socketpair(socket.AF_UNIX, socket.SOCK_STREAM)
    return Channel(a), b


class StatusHeader:
    """Typed view of the status words at `address` (a mapped ShmRegion)."""

    def __init__(self, address: int):
        self.addr = address

    def _u32(self, off):
        return ctypes.c_uint32.from_address(self.addr + off)

    def _u64(self, off):
        return ctypes.c_uint64.from_address(self.addr + off)

    def format(self, pid: int):
        ctypes.memset(self.addr, 0, HEADER_BYTES)
        self._u32(OFF_PROTOCOL).value = PROTOCOL
        self._u32(OFF_PID).value = pid
        self._u32(OFF_MAGIC).value = MAGIC

    def valid(self) -> bool:
        return self._u32(OFF_MAGIC).value == MAGIC and self._u32(OFF_PROTOCOL).value == PROTOCOL

    # runner side
    def set_pid(self, pid: int):
        self._u32(OFF_PID).value = pid

    def beat(self):
        self._u64(OFF_HEARTBEAT).value = time.monotonic_ns()

    def set_step(self, n: int):
        self._u64(OFF_STEP).value = n

    def set_state(self, state: str):
        self._u32(OFF_STATE).value = STATES.index(state)

    def set_pending(self, pending: bool):
        self._u32(OFF_PENDING).value = 1 if pending else 0

    def set_error(self, code: int):
        self._u32(OFF_ERROR).value = code

    # daemon side
    @property
    def pid(self) -> int:
        return self._u32(OFF_PID).value

    @property
    def heartbeat_ns(self) -> int:
        return self._u64(OFF_HEARTBEAT).value

    @property
    def step(self) -> int:
        return self._u64(OFF_STEP).value

    @property
    def state(self) -> str:
        i = self._u32(OFF_STATE).value
        return STATES[i] if i < len(STATES) else "failed"

    @property
    def pending(self) -> bool:
        return bool(self._u32(OFF_PENDING).value)

    @property
    def error(self) -> int:
        return self._u32(OFF_ERROR).value
