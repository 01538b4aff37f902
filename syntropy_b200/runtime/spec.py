"""Speculative decoding: drafters and the exact acceptance step.

A verify step feeds each running sequence's last token plus g drafted tokens as g+1 rows
at consecutive positions (KV written for all of them); the target logits of those rows go
to VerifyAccept (csrc/cuda/sampler.cu), which keeps the drafts the target distribution
agrees with and emits one more token, so every step yields 1..g+1 tokens and the output
distribution is exactly the target's.  Rejected positions' KV is simply overwritten later
(their positions exceed the sequence length).
Reference: plan/rfcs/RFC-0012-execution-scheduler.md :544-630 (verify windows, exact
acceptance); drafts from MTP heads, draft models or prompt lookup.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .._ext import ext


class NgramDrafter:
    """Prompt-lookup drafting: find the most recent earlier occurrence of the last n tokens
    in the sequence's own history and propose what followed it."""

    def __init__(self, n: int = 3):
        self.n = n

    def propose(self, history: list[int], g: int) -> list[int]:
        for n in range(min(self.n, len(history) - 1), 0, -1):
            key = history[-n:]
            for i in range(len(history) - n - 1, -1, -1):
                if history[i:i + n] == key:
                    cont = history[i + n:i + n + g]
                    if cont:
                        return (cont + [cont[-1]] * g)[:g]
        return [history[-1]] * g


@dataclass
class SpecConfig:
    gamma: int = 2
    drafter: object = None

    def __post_init__(self):
        if self.drafter is None:
            self.drafter = NgramDrafter()


def verify(logits, drafts, temperature, top_k, top_p, seed, stream, counter):
    """Device or host acceptance; returns (tokens [S, g+1], n_accept [S]) on the host and
    advances `counter` (host tensor) by the draws taken."""
    if logits.is_cuda:
        dev = logits.device
        S, g = drafts.shape
        out = torch.empty(S, g + 1, dtype=torch.int32, device=dev)
        nacc = torch.empty(S, dtype=torch.int32, device=dev)
        ctr = counter.to(dev)
        ext().verify_accept(logits.contiguous(), drafts.to(dev, torch.int32).contiguous(), temperature.to(dev),
                            top_k.to(dev), top_p.to(dev), seed.to(dev), stream.to(dev), ctr, out, nacc)
        counter.copy_(ctr.cpu())
        return out.cpu(), nacc.cpu()
    from .sampling_ref import verify_ref
    return verify_ref(logits, drafts, temperature, top_k, top_p, seed, stream, counter)
