"""Pipeline parallelism: contiguous layer ranges per stage, hidden states handed from stage
to stage with NCCL point-to-point send/recv (gloo on CPU), the last stage samples and
broadcasts the tokens so every stage's scheduler advances identically.  Prefill is
pipelined over sequence groups with asynchronous isend/irecv (ModelRunner.prefill).  Decode
keeps one hand-off per step: a decode stage's time is the stream of its weights, so splitting
the batch into micro-batches would re-read those weights once per micro-batch and trade the
pipeline's idle time for the same amount of extra weight traffic.
Reference: RFC-0001 :1832-1899 (ring of stages, head embeds, tail samples), ADR-0006.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .dist import DistContext


class PPGroup:
    def __init__(self, ctx: DistContext, n_stages: int, stage: int, n_layers: int, group=None, ranks=None):
        self.ctx = ctx
        self.n_stages, self.stage = n_stages, stage
        self.ranks = ranks or list(range(n_stages))  # global rank of each stage (same TP index)
        self.group = group if group is not None else ctx.group
        per = (n_layers + n_stages - 1) // n_stages
        self.layer_range = (stage * per, min(n_layers, (stage + 1) * per))

    @property
    def first(self) -> bool:
        return self.stage == 0

    @property
    def last(self) -> bool:
        return self.stage == self.n_stages - 1

    def recv_hidden(self, x: torch.Tensor):
        dist.recv(x, src=self.ranks[self.stage - 1], group=self.group)

    def send_hidden(self, x: torch.Tensor):
        dist.send(x.contiguous(), dst=self.ranks[self.stage + 1], group=self.group)

    def irecv_hidden(self, x: torch.Tensor):
        """Posts the receive of the previous stage's hidden states; returns the request."""
        return dist.irecv(x, src=self.ranks[self.stage - 1], group=self.group)

    def isend_hidden(self, x: torch.Tensor):
        """Starts the send to the next stage (x must stay alive until the request completes)."""
        return dist.isend(x.contiguous(), dst=self.ranks[self.stage + 1], group=self.group)

    def broadcast_tokens(self, toks: torch.Tensor) -> torch.Tensor:
        dist.broadcast(toks, src=self.ranks[-1], group=self.group)
        return toks
