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

    def propose_batch(self, histories: list[list[int]], g: int) -> list[list[int]]:
        """Drafts of every running sequence in one native scan (same rule as `propose`)."""
        return ext().ngram_propose(histories, self.n, g)

    def propose(self, history: list[int], g: int) -> list[int]:
        for n in range(min(self.n, len(history) - 1), 0, -1):
            key = history[-n:]
            for i in range(len(history) - n - 1, -1, -1):
                if history[i:i + n] == key:
                    cont = history[i + n:i + n + g]
                    if cont:
                        return (cont + [cont[-1]] * g)[:g]
        return [history[-1]] * g


class DraftModelDrafter:
    """Drafts with a smaller model of the same vocabulary (reference `DraftSource::DraftModel`,
    crates/core/src/plan/speculative.rs): its own runner and paged KV cache.  Per sequence it
    remembers the tokens its cache holds; on each window it keeps the longest prefix that still
    matches the sequence (rejected drafts are overwritten), feeds the rest as one prefill chunk
    after that prefix, then extends greedily one token at a time for the remaining drafts."""
    stateful = True

    def __init__(self, runner, temperature: float = 0.0):
        self.r = runner
        self.fed: dict = {}     # key -> tokens whose K/V the draft cache holds, in order
        self.blocks: dict = {}  # key -> the sequence's pages in the draft cache
        # > 0: drafts are sampled from softmax(draft logits / temperature) and the verify step
        # applies the stochastic-draft rule with those distributions; 0: greedy point masses
        self.temperature = temperature
        self.stochastic = temperature > 0

    def _pick(self, logits: torch.Tensor, gen) -> tuple[int, torch.Tensor | None]:
        if not self.stochastic:
            return int(logits.argmax()), None
        q = torch.softmax(logits.float() / self.temperature, -1)
        return int(torch.multinomial(q.cpu(), 1, generator=gen)), q.cpu()

    def _feed(self, key, toks: list[int], start: int) -> torch.Tensor:
        """K/V for toks at positions start.. (after the cached prefix); returns the next-token logits."""
        r, kv = self.r, self.r.kv
        blocks = self.blocks.setdefault(key, [])
        kv.ensure(blocks, start + len(toks))
        pos = list(range(start, start + len(toks)))
        slots = [kv.slot(blocks, p) for p in pos]
        logits = r.prefill(torch.tensor(toks), torch.tensor(pos), torch.tensor(slots, dtype=torch.int64),
                           [0, len(toks)], [(list(blocks), start)] if start else None, block_lists=[list(blocks)])
        return logits[0]

    def propose(self, history: list[int], g: int, key=None, seed: int = 0):
        """g drafts after history: greedy tokens, or (stochastic) tokens sampled from the
        draft model with their distributions [g, V] (returned as (tokens, probs)); the
        draws are keyed by (seed, position), so a window is reproducible."""
        fed = self.fed.get(key, [])
        c = 0
        lim = min(len(fed), len(history) - 1)  # the last token is always fed again (its logits)
        while c < lim and fed[c] == history[c]:
            c += 1
        gen = None
        if self.stochastic:
            gen = torch.Generator().manual_seed((seed * 1000003 + len(history)) & ((1 << 63) - 1))
        nxt, q = self._pick(self._feed(key, history[c:], c), gen)
        drafts, probs = [nxt], [q]
        fed = list(history)
        for _ in range(g - 1):
            nxt, q = self._pick(self._feed(key, [drafts[-1]], len(fed)), gen)
            fed.append(drafts[-1])
            drafts.append(nxt)
            probs.append(q)
        self.fed[key] = fed
        return (drafts, torch.stack(probs)) if self.stochastic else drafts

    def release(self, key):
        """Forget a finished sequence and return its draft pages."""
        self.fed.pop(key, None)
        blocks = self.blocks.pop(key, None)
        if blocks:
            self.r.kv.release(blocks)


class MTPDrafter:
    """Drafts with the model's multi-token-prediction head (DeepSeek-V3 style): one token per
    step from the final residual of the last accepted position and the token after it.  The
    engine calls `after_prefill` and `after_verify` to keep the MTP block's KV and the next
    draft per sequence."""
    gamma_max = 1

    def __init__(self, runner):
        self.runner = runner

    def _run(self, rows):
        if not rows:
            return
        kv = self.runner.kv
        xs = torch.stack([r[1] for r in rows])
        toks = torch.tensor([r[2] for r in rows], dtype=torch.int32)
        pos = torch.tensor([r[3] for r in rows], dtype=torch.int64)
        for s, _, _, p in rows:
            kv.ensure(s.blocks, p + 2)
        slots = torch.tensor([kv.slot(s.blocks, p) for s, _, _, p in rows], dtype=torch.int64)
        drafts = self.runner.mtp_forward(xs, toks, pos, slots, [list(s.blocks) for s, _, _, _ in rows])
        for (s, _, _, _), d in zip(rows, drafts.tolist()):
            if s.mtp_draft is not None:
                s.mtp_draft = [d]

    def after_prefill(self, seqs, x_rows, cu):
        rows_fill = []
        for i, s in enumerate(seqs):
            s.mtp_draft = []
            a, b = cu[i], cu[i + 1]
            st = s.cached_tokens
            # MTP KV for prompt positions st+1..P-1 from (x_{j-1}, t_j), then the first draft
            for j in range(max(1, st + 1), len(s.prompt)):
                rows_fill.append((s, x_rows[a + j - 1 - st], s.prompt[j], j))
            rows_fill.append((s, x_rows[b - 1], s.output[-1], len(s.prompt)))
        self._run(rows_fill)

    def after_verify(self, items):
        """items: (seq, final residual of the last accepted row, its position)."""
        self._run([(s, x, s.output[-1], p + 1) for s, x, p in items if s.status != "finished"])

    def propose(self, history, g):
        raise RuntimeError("MTPDrafter drafts per sequence state")


@dataclass
class SpecConfig:
    gamma: int = 2
    drafter: object = None
    # adaptive pause: when fewer than min_accept of the last `window` drafted tokens were
    # accepted, the engine takes `pause_steps` plain decode steps (a verify window costs about
    # g + 1 rows of work for one token when nothing is accepted), then drafts again.  Not for
    # MTP (its drafts come from the verify pass) nor under lockstep ranks.  min_accept 0: off.
    min_accept: float = 0.1
    window: int = 256
    pause_steps: int = 32

    def __post_init__(self):
        if self.drafter is None:
            self.drafter = NgramDrafter()
        if isinstance(self.drafter, MTPDrafter):
            self.gamma = 1


def verify(logits, drafts, temperature, top_k, top_p, seed, stream, counter, draft_probs=None):
    """Device or host acceptance; returns (tokens [S, g+1], n_accept [S]) on the host and
    advances `counter` (host tensor) by the draws taken.  draft_probs [S, g, V]: the
    distributions stochastic drafts were sampled from (None: point-mass drafts)."""
    if logits.is_cuda:
        dev = logits.device
        S, g = drafts.shape
        out = torch.empty(S, g + 1, dtype=torch.int32, device=dev)
        nacc = torch.empty(S, dtype=torch.int32, device=dev)
        ctr = counter.to(dev)
        dp = draft_probs.to(dev, torch.float32).contiguous() if draft_probs is not None else \
            torch.empty(0, dtype=torch.float32, device=dev)
        ext().verify_accept(logits.contiguous(), drafts.to(dev, torch.int32).contiguous(), temperature.to(dev),
                            top_k.to(dev), top_p.to(dev), seed.to(dev), stream.to(dev), ctr, out, nacc, dp)
        counter.copy_(ctr.cpu())
        return out.cpu(), nacc.cpu()
    from .sampling_ref import verify_ref
    return verify_ref(logits, drafts, temperature, top_k, top_p, seed, stream, counter, draft_probs)
