"""Membership: a sans-I/O failure detector of one node (SWIM-style heartbeats with
incarnation numbers) and a coordinator lease with fencing terms.

Membership: every `period_s` a node sends a heartbeat (its incarnation, and the members it
currently suspects) to each peer.  A peer silent for `suspect_after_s` becomes Suspect, for
`fail_after_s` Failed; a heartbeat from a Suspect (or Failed) member makes it Alive again.  A
node that learns it is suspected raises its incarnation, so its next heartbeats refute the
suspicion everywhere.  State changes come out as cluster-log events (member_suspect,
member_leave, member_join).  Defaults are the LAN timings (1 s, 3 s, 7 s).

Lease: one coordinator at a time.  A candidate asks every member for term + 1; a member grants
only if it sees no live lease (its last renewal from a holder is older than `lease_s`) and the
term is higher than any it granted; with a majority of grants the candidate holds the lease.
The holder renews every `renew_s`; a member acknowledges a renewal of the term it granted.
The holder steps down `lease_s - margin_s` after the send time of the last renewal round that
a majority acknowledged, which is never later than when any member of that majority would
grant a new term: two holders never overlap, and a partitioned minority holder steps down.

Both are protocol cores driven by explicit time: `tick(now)` and `on_message(now, src, msg)`
return the messages to send and the events raised.  Reference: crates/cluster/src/ (config
sections membership / recovery), RFC-0032 summary (SWIM membership, coordinator lease with
pre-vote, terms), plan/00-vision-and-scope.md:297 (SC-25: Suspect after 3 missed heartbeats,
NodeFailed <= 8 s).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field


class Status(enum.Enum):
    ALIVE = "alive"
    SUSPECT = "suspect"
    FAILED = "failed"


@dataclass
class MembershipConfig:
    period_s: float = 1.0
    suspect_after_s: float = 3.0
    fail_after_s: float = 7.0


@dataclass
class _Peer:
    status: Status = Status.ALIVE
    last_seen: float = 0.0
    incarnation: int = 0


class Membership:
    def __init__(self, me: str, peers: list[str], cfg: MembershipConfig | None = None, now: float = 0.0):
        self.me = me
        self.cfg = cfg or MembershipConfig()
        self.incarnation = 0
        self.peers = {p: _Peer(last_seen=now) for p in peers if p != me}
        self._next_beat = now

    def tick(self, now: float) -> tuple[list, list]:
        """(messages [(dst, msg)], events [(kind, node)]) due at `now`."""
        out, events = [], []
        for name, p in self.peers.items():
            silent = now - p.last_seen
            if p.status == Status.ALIVE and silent >= self.cfg.suspect_after_s:
                p.status = Status.SUSPECT
                events.append(("member_suspect", name))
            if p.status == Status.SUSPECT and silent >= self.cfg.fail_after_s:
                p.status = Status.FAILED
                events.append(("member_leave", name))
        if now >= self._next_beat:
            self._next_beat = now + self.cfg.period_s
            suspects = sorted(n for n, p in self.peers.items() if p.status != Status.ALIVE)
            msg = {"type": "hb", "inc": self.incarnation, "suspects": suspects}
            out = [(n, msg) for n in self.peers]
        return out, events

    def on_message(self, now: float, src: str, msg: dict) -> list:
        """Events raised by a heartbeat from src."""
        if msg.get("type") != "hb" or src not in self.peers:
            return []
        events = []
        p = self.peers[src]
        if msg["inc"] >= p.incarnation:
            p.incarnation = msg["inc"]
            p.last_seen = now
            if p.status != Status.ALIVE:
                events.append(("member_join", src))
                p.status = Status.ALIVE
        if self.me in msg.get("suspects", ()):
            self.incarnation += 1  # refute: the next heartbeats carry a newer incarnation
        return events

    def status(self, name: str) -> Status:
        return self.peers[name].status


@dataclass
class LeaseConfig:
    lease_s: float = 10.0
    renew_s: float = 2.0
    margin_s: float = 1.0


@dataclass
class Lease:
    me: str
    members: list
    cfg: LeaseConfig = field(default_factory=LeaseConfig)
    term: int = 0                 # highest term granted or held here
    granted_to: str | None = None
    last_renew_seen: float = -1e18
    holding: bool = False
    held_term: int = 0
    _grants: set = field(default_factory=set)
    _want_term: int = 0
    _rounds: dict = field(default_factory=dict)   # renewal round -> (send time, acks)
    _round: int = 0
    _valid_until: float = -1e18
    _next_renew: float = 0.0
    _campaign_t: float = 0.0

    @property
    def majority(self) -> int:
        return len(self.members) // 2 + 1

    def campaign(self, now: float) -> list:
        """Ask every member for term + 1 (this node grants itself first if it can)."""
        self._want_term = self.term + 1
        self._grants = set()
        self._campaign_t = now  # every grant of this campaign happens after this instant
        out = [(m, {"type": "lease_req", "term": self._want_term, "cand": self.me}) for m in self.members
               if m != self.me]
        self._maybe_grant(now, self._want_term, self.me, self_vote=True)
        return out

    def _live_lease(self, now: float) -> bool:
        return now - self.last_renew_seen < self.cfg.lease_s

    def _maybe_grant(self, now, term, cand, self_vote=False) -> bool:
        if term > self.term and (not self._live_lease(now) or self.granted_to == cand):
            self.term = term
            self.granted_to = cand
            if self_vote:
                # a node's vote for itself is not a lease it has seen: it stays free to grant a
                # later, higher term to another candidate if its own campaign fails
                self._grants.add(self.me)
            else:
                self.last_renew_seen = now
            return True
        return False

    def tick(self, now: float) -> tuple[list, list]:
        out, events = [], []
        if self.holding and now >= self._valid_until:
            self.holding = False
            events.append(("lease_lost", self.held_term))
        if self.holding and now >= self._next_renew:
            self._next_renew = now + self.cfg.renew_s
            self._round += 1
            self._rounds[self._round] = (now, {self.me})
            self.last_renew_seen = now
            out = [(m, {"type": "lease_renew", "term": self.held_term, "round": self._round}) for m in self.members
                   if m != self.me]
            self._rounds = {r: v for r, v in self._rounds.items() if r > self._round - 8}
        return out, events

    def on_message(self, now: float, src: str, msg: dict) -> tuple[list, list]:
        t = msg.get("type")
        out, events = [], []
        if t == "lease_req":
            ok = self._maybe_grant(now, msg["term"], msg["cand"])
            out.append((src, {"type": "lease_grant" if ok else "lease_deny", "term": msg["term"]}))
        elif t == "lease_grant" and msg["term"] == self._want_term and not self.holding:
            self._grants.add(src)
            if len(self._grants) >= self.majority and self.term == self._want_term:
                self.holding = True
                self.held_term = self._want_term
                # a granting member treats the lease as live from its grant, which came after the
                # campaign started: counting from the start keeps the holder's view the shorter
                self._valid_until = self._campaign_t + self.cfg.lease_s - self.cfg.margin_s
                self._next_renew = now
                events.append(("lease_acquired", self.held_term))
        elif t == "lease_renew":
            if msg["term"] >= self.term:
                self.term = msg["term"]
                self.granted_to = src
                self.last_renew_seen = now
                out.append((src, {"type": "lease_ack", "term": msg["term"], "round": msg["round"]}))
        elif t == "lease_ack" and self.holding and msg["term"] == self.held_term:
            r = self._rounds.get(msg["round"])
            if r is not None:
                sent, acks = r
                acks.add(src)
                if len(acks) >= self.majority:
                    self._valid_until = max(self._valid_until, sent + self.cfg.lease_s - self.cfg.margin_s)
        return out, events
