"""Data-plane payloads on the 64-byte frame header: the native codecs of
csrc/include/syn/payload.h, with Python-side conveniences.

* Activation: hidden-state rows passed from one pipeline stage to the next (kind prefill /
  decode / verify / replay / canary), the spans of sequences they belong to, and a chunk split
  into parts at row boundaries when it exceeds a frame size limit.
* Token: sampled tokens per sequence, with a finished flag and a finish-reason code.
* Collective: one member's part of a group reduction or gather (phase, layer, member, rows).
* EP dispatch / combine: rows sent to the owner of some of their experts with a route record
  per row (source row, experts, weights), and the owner's weighted f32 sums sent back.

Reference: crates/net/src/frame/activation.rs:82-482, crates/net/src/frame/token.rs,
crates/net/src/frame/collective.rs:1-40, crates/net/src/frame/ep.rs:1-50 (semantics; the
extension and payload layouts here are this framework's own).
"""
from __future__ import annotations

import torch

from .._ext import ext

KINDS = {"prefill": 1, "decode": 2, "verify": 3, "replay": 4, "canary": 5}
REASONS = {None: 0, "stop": 1, "length": 2, "cancelled": 3}
FINISHED = 1


class FrameError(ValueError):
    """A frame failed its checks (code from the native decoder: 1 short, 2 magic, 3 header CRC,
    4 payload CRC, 5 extension alignment, 10 type, 11 dtype, 12 length, 13 span)."""

    def __init__(self, code: int):
        super().__init__(f"frame rejected (code {code})")
        self.code = code


def encode_activation(rows: torch.Tensor, spans: list[tuple[int, int, int, int]], kind: str = "decode",
                      from_stage: int = 0, to_stage: int = 1, step: int = 0, chan_seq: int = 0,
                      instance: int = 0, streams: int = 1, kind_arg: int = 0, kind_flags: int = 0,
                      part: tuple[int, int] = (0, 1)) -> bytes:
    """rows: [n, streams * hidden] f32 or bf16; spans: (sequence id, first position, positions,
    first row)."""
    r = rows.detach().to("cpu").contiguous()
    return ext().activation_encode({"instance": instance, "step": step, "chan_seq": chan_seq},
                                   {"from_stage": from_stage, "to_stage": to_stage, "kind": KINDS[kind],
                                    "streams": streams, "kind_arg": kind_arg, "kind_flags": kind_flags,
                                    "part_index": part[0], "part_count": part[1]}, list(spans), r)


def decode_activation(buf: bytes) -> tuple[dict, dict, list, torch.Tensor]:
    rc, spec, hdr, spans, rows = ext().activation_decode(buf)
    if rc:
        raise FrameError(rc)
    return spec, hdr, [tuple(s) for s in spans], rows


def split_activation(rows: torch.Tensor, spans: list, max_rows: int, **kw) -> list[bytes]:
    """A chunk as parts of at most max_rows rows, split at row boundaries; each part carries
    the pieces of the spans that fall in its rows (row offsets relative to the part)."""
    n = rows.shape[0]
    bounds = list(range(0, n, max_rows)) or [0]
    out = []
    for i, a in enumerate(bounds):
        b = min(n, a + max_rows)
        part_spans = []
        for seq, first, npos, r0 in spans:
            lo, hi = max(a, r0), min(b, r0 + npos)
            if lo < hi:
                part_spans.append((seq, first + (lo - r0), hi - lo, lo - a))
        out.append(encode_activation(rows[a:b], part_spans, part=(i, len(bounds)), **kw))
    return out


def join_activation(parts: list[bytes]) -> tuple[dict, torch.Tensor, list]:
    """Reassembles parts (in any order) into (header of part 0, rows, spans with absolute rows)."""
    dec = sorted((decode_activation(p) for p in parts), key=lambda d: d[1]["part_index"])
    if not dec or len(dec) != dec[0][1]["part_count"] or \
            [d[1]["part_index"] for d in dec] != list(range(len(dec))):
        raise FrameError(12)
    rows, spans, base = [], {}, 0
    for _, hdr, sp, r in dec:
        for seq, first, npos, r0 in sp:
            if seq in spans:
                s0 = spans[seq]
                spans[seq] = (seq, s0[1], s0[2] + npos, s0[3])
            else:
                spans[seq] = (seq, first, npos, base + r0)
        rows.append(r)
        base += r.shape[0]
    return dec[0][1], torch.cat(rows, 0), list(spans.values())


def encode_tokens(entries: list[tuple[int, list[int], bool, str | None]], step: int = 0, chan_seq: int = 0,
                  instance: int = 0) -> bytes:
    """entries: (sequence id, new tokens, finished, finish reason)."""
    return ext().token_encode({"instance": instance, "step": step, "chan_seq": chan_seq},
                              [(seq, list(map(int, toks)), (FINISHED if fin else 0) | (REASONS[reason] << 8))
                               for seq, toks, fin, reason in entries])


def decode_tokens(buf: bytes) -> tuple[dict, list]:
    rc, spec, entries = ext().token_decode(buf)
    if rc:
        raise FrameError(rc)
    inv = {v: k for k, v in REASONS.items()}
    return spec, [(seq, toks, bool(fl & FINISHED), inv.get(fl >> 8)) for seq, toks, fl in entries]


PHASES = {"attn_allreduce": 1, "ffn_allreduce": 2, "exit_gather": 3, "logits_gather": 4}


def encode_collective(rows: torch.Tensor, phase: str, member: int, n_members: int, layer: int,
                      row_offset: int = 0, epoch: int = 0, step: int = 0, chan_seq: int = 0,
                      instance: int = 0) -> bytes:
    """rows: [n, width] f32 or bf16, this member's part (rows from row_offset)."""
    return ext().collective_encode({"instance": instance, "step": step, "chan_seq": chan_seq},
                                   {"phase": PHASES[phase], "member": member, "n_members": n_members,
                                    "layer": layer, "row_offset": row_offset, "epoch": epoch},
                                   rows.detach().to("cpu").contiguous())


def decode_collective(buf: bytes) -> tuple[dict, dict, torch.Tensor]:
    rc, spec, hdr, rows = ext().collective_decode(buf)
    if rc:
        raise FrameError(rc)
    inv = {v: k for k, v in PHASES.items()}
    hdr["phase"] = inv.get(hdr["phase"], hdr["phase"])
    return spec, hdr, rows


def reduce_collective(frames: list[bytes]) -> torch.Tensor:
    """Sum of the members' rows of one reduction in member order (identical bits whatever
    order the frames arrived in)."""
    dec = sorted((decode_collective(f) for f in frames), key=lambda d: d[1]["member"])
    n = dec[0][1]["n_members"] if dec else 0
    if [d[1]["member"] for d in dec] != list(range(n)) or len({d[1]["layer"] for d in dec}) != 1:
        raise FrameError(13)
    acc = dec[0][2].float().clone()
    for _, _, r in dec[1:]:
        acc += r.float()
    return acc


def encode_ep_dispatch(rows: torch.Tensor, routes: list[tuple[int, list[tuple[int, float]]]], src_rank: int,
                       dst_rank: int, layer: int, top_k: int, epoch: int = 0, step: int = 0, chan_seq: int = 0,
                       instance: int = 0) -> bytes:
    """rows [n, hidden] (bf16 or f32); routes: per row (source row, [(expert, weight)])."""
    return ext().ep_dispatch_encode({"instance": instance, "step": step, "chan_seq": chan_seq},
                                    {"src_rank": src_rank, "dst_rank": dst_rank, "layer": layer, "top_k": top_k,
                                     "epoch": epoch},
                                    [(int(r), [(int(e), float(w)) for e, w in rt]) for r, rt in routes],
                                    rows.detach().to("cpu").contiguous())


def decode_ep_dispatch(buf: bytes) -> tuple[dict, dict, list, torch.Tensor]:
    rc, spec, hdr, routes, rows = ext().ep_dispatch_decode(buf)
    if rc:
        raise FrameError(rc)
    return spec, hdr, [(r, [tuple(x) for x in rt]) for r, rt in routes], rows


def encode_ep_combine(rows: torch.Tensor, row_ids: list[int], src_rank: int, dst_rank: int, layer: int,
                      epoch: int = 0, step: int = 0, chan_seq: int = 0, instance: int = 0) -> bytes:
    """rows [n, hidden] f32: the owner's weighted sum over its experts for each source row."""
    return ext().ep_combine_encode({"instance": instance, "step": step, "chan_seq": chan_seq},
                                   {"src_rank": src_rank, "dst_rank": dst_rank, "layer": layer, "epoch": epoch},
                                   [int(i) for i in row_ids], rows.detach().to("cpu").float().contiguous())


def decode_ep_combine(buf: bytes) -> tuple[dict, dict, list, torch.Tensor]:
    rc, spec, hdr, ids, rows = ext().ep_combine_decode(buf)
    if rc:
        raise FrameError(rc)
    return spec, hdr, list(ids), rows
