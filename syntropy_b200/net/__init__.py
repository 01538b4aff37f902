"""Data-plane transport across hosts: the 64-byte frame codec (native, csrc/include/syn/
frame.h) over TCP with per-channel sequence numbers and credit flow control
(reference: crates/net/src/transport/{mod.rs:120,core.rs:93-215,tcp.rs})."""
from .tcp import FrameType, TcpChannel, TcpListener  # noqa: F401
