"""Error taxonomy (reference: crates/core/src/error.rs:31-58).  Every error carries a class
(what kind of failure, which decides retry/abandon/restart policy), a domain and a code."""
from __future__ import annotations

import enum


class ErrorClass(enum.Enum):
    INVALID_REQUEST = "invalid_request"   # bad client input
    UNSUPPORTED = "unsupported"           # op, dtype or feature missing on this device/build
    CAPACITY = "capacity"                 # VRAM, pinned RAM, KV pool or admission limit
    TRANSIENT = "transient"               # momentary: would-block, one lost message
    LINK = "link"                         # transport/NVLink failure on one link
    DEVICE = "device"                     # device fault or sticky driver error
    INTEGRITY = "integrity"               # hash mismatch, corrupt file
    CORRECTNESS = "correctness"           # parity or canary failure
    DRIFT = "drift"                       # measured costs no longer match the plan
    TIMEOUT = "timeout"                   # deadline passed / progress stalled (bounded waits)
    AUTH = "auth"
    CANCELLED = "cancelled"
    INTERNAL = "internal"

    @property
    def retryable(self) -> bool:
        return self in (ErrorClass.TRANSIENT, ErrorClass.LINK, ErrorClass.TIMEOUT)

    @property
    def http_status(self) -> int:
        return {ErrorClass.INVALID_REQUEST: 400, ErrorClass.UNSUPPORTED: 400, ErrorClass.CAPACITY: 503,
                ErrorClass.AUTH: 401, ErrorClass.CANCELLED: 499, ErrorClass.TIMEOUT: 504}.get(self, 500)


class Domain(enum.IntEnum):
    CORE = 0
    KERNELS = 1
    IO = 2
    NET = 3
    SCHED = 4
    API = 5
    TIER = 6
    CLUSTER = 7


class SynError(Exception):
    def __init__(self, cls: ErrorClass, message: str, domain: Domain = Domain.CORE, code: int = 0):
        super().__init__(message)
        self.cls, self.domain, self.code = cls, domain, code

    def to_json(self) -> dict:
        return {"type": self.cls.value, "domain": self.domain.name.lower(), "code": self.code, "message": str(self)}


# Kernel-domain codes used by the bounded device waits (reference: RFC-0040 `DoorbellTimeout`).
KERNELS_DOORBELL_TIMEOUT = 11
KERNELS_PEER_TIMEOUT = 12
KERNELS_PIPELINE_TIMEOUT = 13


def device_status_error(status: int) -> SynError | None:
    """Maps the int32 status word written by the kernels' bounded waits to an error."""
    if status == 0:
        return None
    if status & 0b11:
        return SynError(ErrorClass.TIMEOUT, f"peer flag wait timed out (status=0x{status:x})", Domain.KERNELS,
                        KERNELS_PEER_TIMEOUT)
    if status & (1 << 4):
        return SynError(ErrorClass.TIMEOUT, f"GEMM pipeline wait timed out (status=0x{status:x})", Domain.KERNELS,
                        KERNELS_PIPELINE_TIMEOUT)
    return SynError(ErrorClass.DEVICE, f"device status 0x{status:x}", Domain.KERNELS, 0)
