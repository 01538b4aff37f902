"""LAN pairing: the joiner's commitment to its nonce, the keyholder's challenge, the reveal, and
the six-digit short authentication string (SAS) both sides show for the user to compare.

Order of the fields (the joiner reveals only after the keyholder's nonce has arrived, so neither
side picks its nonce knowing the other's; a relaying attacker matches the two codes with
probability about 1e-6 per attempt):

1. joiner -> keyholder: commit = BLAKE3("syntropy-sas-commit-v1" | joiner | nonce_c)  (32 B)
2. keyholder -> joiner: nonce_k                                                      (16 B)
3. joiner -> keyholder: nonce_c; the keyholder checks it opens the commitment         (16 B)

SAS = u32_le(BLAKE3("syntropy-sas-v1" | cluster_id | joiner | keyholder | nonce_c | nonce_k)[0:4])
mod 10^6, shown as two groups of three digits with leading zeros.  Every field has a fixed
length, so the concatenations are unambiguous.  The domain strings, field order and reduction
are the wire protocol and match the reference's frozen vectors (crates/cluster/src/pairing.rs:
28-100), so nodes of either implementation pair with each other.

`Joiner` and `Keyholder` are sans-I/O state machines over those three messages.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

from .._ext import ext

COMMIT_CONTEXT = b"syntropy-sas-commit-v1"
SAS_CONTEXT = b"syntropy-sas-v1"
SAS_CODES = 1_000_000
NONCE_BYTES, ID_BYTES = 16, 32


def blake3(data: bytes) -> bytes:
    return ext().blake3(bytes(data))


def _check(name: str, b: bytes, n: int):
    if len(b) != n:
        raise ValueError(f"{name}: {len(b)} bytes, expected {n}")


def commitment(joiner: bytes, nonce_c: bytes) -> bytes:
    _check("joiner", joiner, ID_BYTES)
    _check("nonce_c", nonce_c, NONCE_BYTES)
    return blake3(COMMIT_CONTEXT + joiner + nonce_c)


def opens(commit: bytes, joiner: bytes, nonce_c: bytes) -> bool:
    """Whether `nonce_c` opens `commit` for `joiner` (all public once revealed: no constant-time
    comparison needed)."""
    return commitment(joiner, nonce_c) == commit


def sas_digest(cluster_id: bytes, joiner: bytes, keyholder: bytes, nonce_c: bytes, nonce_k: bytes) -> bytes:
    for name, b, n in (("cluster_id", cluster_id, ID_BYTES), ("joiner", joiner, ID_BYTES),
                       ("keyholder", keyholder, ID_BYTES), ("nonce_c", nonce_c, NONCE_BYTES),
                       ("nonce_k", nonce_k, NONCE_BYTES)):
        _check(name, b, n)
    return blake3(SAS_CONTEXT + cluster_id + joiner + keyholder + nonce_c + nonce_k)


@dataclass(frozen=True)
class Sas:
    value: int

    @classmethod
    def from_digest(cls, digest: bytes) -> "Sas":
        return cls(int.from_bytes(digest[:4], "little") % SAS_CODES)

    def __str__(self) -> str:
        return f"{self.value // 1000:03d} {self.value % 1000:03d}"


def sas(cluster_id: bytes, joiner: bytes, keyholder: bytes, nonce_c: bytes, nonce_k: bytes) -> Sas:
    return Sas.from_digest(sas_digest(cluster_id, joiner, keyholder, nonce_c, nonce_k))


class PairingError(Exception):
    pass


class Joiner:
    """request() -> commit; on_challenge(nonce_k) -> nonce_c (the reveal); code() afterwards."""

    def __init__(self, cluster_id: bytes, joiner: bytes, keyholder: bytes, nonce_c: bytes | None = None):
        self.cluster_id, self.joiner, self.keyholder = cluster_id, joiner, keyholder
        self.nonce_c = nonce_c if nonce_c is not None else os.urandom(NONCE_BYTES)
        self.nonce_k = None
        self.state = "start"

    def request(self) -> bytes:
        if self.state != "start":
            raise PairingError(f"request in state {self.state}")
        self.state = "committed"
        return commitment(self.joiner, self.nonce_c)

    def on_challenge(self, nonce_k: bytes) -> bytes:
        if self.state != "committed":
            raise PairingError(f"challenge in state {self.state}")  # reveal only after our commit
        _check("nonce_k", nonce_k, NONCE_BYTES)
        self.nonce_k = nonce_k
        self.state = "revealed"
        return self.nonce_c

    def code(self) -> Sas:
        if self.state != "revealed":
            raise PairingError("no code before the reveal")
        return sas(self.cluster_id, self.joiner, self.keyholder, self.nonce_c, self.nonce_k)


class Keyholder:
    """on_request(commit) -> nonce_k; on_reveal(nonce_c) checks the commitment; code()."""

    def __init__(self, cluster_id: bytes, keyholder: bytes, joiner: bytes, nonce_k: bytes | None = None):
        self.cluster_id, self.keyholder, self.joiner = cluster_id, keyholder, joiner
        self.nonce_k = nonce_k if nonce_k is not None else os.urandom(NONCE_BYTES)
        self.commit = self.nonce_c = None
        self.state = "start"

    def on_request(self, commit: bytes) -> bytes:
        if self.state != "start":
            raise PairingError(f"request in state {self.state}")
        _check("commit", commit, 32)
        self.commit = commit
        self.state = "challenged"
        return self.nonce_k

    def on_reveal(self, nonce_c: bytes):
        if self.state != "challenged":
            raise PairingError(f"reveal in state {self.state}")
        if not opens(self.commit, self.joiner, nonce_c):
            self.state = "denied"
            raise PairingError("denied: the reveal does not open the commitment")
        self.nonce_c = nonce_c
        self.state = "revealed"

    def code(self) -> Sas:
        if self.state != "revealed":
            raise PairingError("no code before a valid reveal")
        return sas(self.cluster_id, self.joiner, self.keyholder, self.nonce_c, self.nonce_k)
