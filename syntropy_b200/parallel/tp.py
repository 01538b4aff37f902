"""Intra-node tensor parallelism (Megatron column/row split over NVLink).

Column-parallel: qkv (whole KV heads per rank) and gate/up; row-parallel: o_proj and down.
The row-parallel products are reduced by a fused path on GPUs: the GEMV (4-bit weights) or
the tcgen05 GEMM (bf16 weights, csrc/cuda/gemm_bf16_tc.cu) pushes its f32 partial rows from
its epilogue straight into every peer's receive slot over NVLink and the last CTA raises a
flag; the receive kernel sums the N partials in rank order (so every rank holds bitwise
identical residuals, the reference's member-order rule), adds the residual and applies the
next RMSNorm.  The NCCL all-reduce path is the baseline (and the CPU/gloo path).

Reference: plan/rfcs/RFC-0032-distributed-execution.md:372-396 (TP layer, member-order f32
reduction), crates/solver/src/collective.rs:256-333 (one-shot vs ring).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .._ext import ext
from .dist import DistContext
from .symm import SymmetricRegion


def _align(n, a=256):
    return (n + a - 1) // a * a


def gather_vocab_logits(local: torch.Tensor, out: torch.Tensor, gathered: torch.Tensor, group):
    """out [T, V] = concatenation over ranks (rank order) of local [T, V/N] vocab slices."""
    n = dist.get_world_size(group)
    T, vl = local.shape
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered[: n * T], local, group=group)
    else:
        parts = [torch.empty_like(local) for _ in range(n)]
        dist.all_gather(parts, local.contiguous(), group=group)
        torch.cat(parts, 0, out=gathered[: n * T])
    out.copy_(gathered[: n * T].view(n, T, vl).permute(1, 0, 2).reshape(T, n * vl))


class TPGroup:
    def __init__(self, ctx: DistContext, hidden: int, cap: int, n_layers: int, timeout_s: float = 2.0,
                 fused: bool = True, vocab: int = 0):
        """vocab > 0 (a vocab-parallel head with bf16 weights): the LM-head GEMM of each rank
        writes its column slice of the logits straight into every rank's logits buffer, which
        lives in the symmetric region (`logits_view`)."""
        self.ctx = ctx
        self.N, self.rank, self.H, self.cap = ctx.world, ctx.rank, hidden, cap
        self.n_layers = n_layers
        self.fused = fused and ctx.device.type == "cuda"
        self.timeout_ns = int(timeout_s * 1e9)
        self.vocab = vocab if self.fused and vocab % self.N == 0 else 0
        if self.fused:
            area = self.N * cap * hidden * 4
            self.off_recv = [0, _align(area)]
            self.off_flag = [2 * _align(area), 2 * _align(area) + 256, 2 * _align(area) + 512]
            self.off_logits = 2 * _align(area) + 768
            size = self.off_logits + (_align(cap * self.vocab * 4) if self.vocab else 0)
            self.region = SymmetricRegion(ctx, size)
            dev = ctx.device
            self.step_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.done_ctr = torch.zeros(2 * n_layers + 1, dtype=torch.int32, device=dev)
            self._off1 = {}
            # prefill (MiB-scale messages): ordered two-shot all-reduce over a second region
            # holding a partial and a gather buffer of `prefill_rows` rows, plus ready / done
            # flags; sequence numbers come from a host counter (prefill runs eagerly)
            self.prefill_rows = max(256, (64 << 20) // (hidden * 4) // 256 * 256)
            part = _align(self.prefill_rows * hidden * 4)
            self.off_part, self.off_gather = 0, part
            self.off_ready, self.off_done = 2 * part, 2 * part + 256
            self.region2 = SymmetricRegion(ctx, 2 * part + 512)
            self.ts_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
            self.ts_seq = 0

    def step_begin(self):
        if self.fused:
            ext().ep_step_begin(self.step_ctr)

    def logits_view(self, rows: int) -> torch.Tensor:
        """f32 [rows, vocab] logits buffer in the symmetric region (every rank's slices land here)."""
        return self.region.view(self.off_logits, self.cap * self.vocab, torch.float32).view(self.cap, self.vocab)[:rows]

    def gather_logits(self, h, W, logits_rows: int):
        """Vocab-parallel head, fused: this rank's slice of h @ W^T (bf16 W [V/N, H]) goes from the
        GEMM epilogue into columns [rank * V/N, (rank + 1) * V/N) of every rank's logits buffer
        over NVLink; then a bounded wait for every rank's slice.  Returns the logits view."""
        from ..ops.core import _bf16_workspace, gemm_status
        T = h.shape[0]
        vl = W.shape[0]
        seq = 2 * self.n_layers  # the head's flag slot: its own monotone sequence per step
        ws, ctr = _bf16_workspace(h.device, vl, W.shape[1], T)
        ext().gemm_bf16_tp(h, W, self.region.peers, self.off_logits, self.cap, self.vocab, 0, self.off_flag[2],
                           self.rank, self.done_ctr[seq:seq + 1], self.step_ctr, 2 * self.n_layers, seq, ws, ctr,
                           gemm_status(h.device), vl)
        ext().flags_wait(self.region.peers, self.rank, self.off_flag[2], self.step_ctr, 2 * self.n_layers, seq,
                         self.timeout_ns, self.status)
        ops.core._launched(2)
        return self.logits_view(T)

    def _tok_off(self, T, dev):
        t = self._off1.get(T)
        if t is None:
            t = torch.tensor([0, T], dtype=torch.int32, device=dev)
            self._off1[T] = t
        return t

    def row_parallel_reduce(self, which: int, layer: int, x_in, W, x_res, next_norm, h_out, eps):
        """x_res += all_reduce(x_in @ W^T) across ranks; h_out = rmsnorm(x_res) (if next_norm).
        which: 0 = attention output projection, 1 = FFN down projection."""
        T = x_in.shape[0]
        if self.fused:
            seq_layer = 2 * layer + which
            if isinstance(W, torch.Tensor) and W.dtype == torch.bfloat16:
                # bf16 weights: the tcgen05 GEMM pushes each f32 partial row to every peer
                from ..ops.core import _bf16_workspace, gemm_status
                ws, ctr = _bf16_workspace(x_in.device, W.shape[0], W.shape[1], T)
                ext().gemm_bf16_tp(x_in, W, self.region.peers, self.off_recv[which], self.cap, self.H, 0,
                                   self.off_flag[which], self.rank, self.done_ctr[seq_layer:seq_layer + 1],
                                   self.step_ctr, 2 * self.n_layers, seq_layer, ws, ctr, gemm_status(x_in.device), 0)
            elif T >= ops.core._Q4_TC[0] and W.N % 128 == 0 and W.K % 64 == 0:
                # 16-64 rows of 4-bit weights: the tcgen05 decode GEMM pushes each f32 row to every peer
                from ..ops.core import gemm_status
                ext().q4_gemm_dec_tp(x_in, W.qw, W.sm, W.N, W.K, self.region.peers, self.off_recv[which], self.cap,
                                     self.H, self.off_flag[which], self.rank, self.done_ctr[seq_layer:seq_layer + 1],
                                     self.step_ctr, 2 * self.n_layers, seq_layer, gemm_status(x_in.device))
            else:
                from ..ops.core import _ptrs
                qp, sp = _ptrs(W)
                ext().q4_gemv_tp(x_in, qp, sp, self._tok_off(T, x_in.device), W.N, W.K,
                                 self.done_ctr[seq_layer:seq_layer + 1], self.region.peers, self.off_recv[which],
                                 self.cap, self.off_flag[which], self.rank, self.step_ctr, 2 * self.n_layers,
                                 seq_layer)
            ext().tp_reduce_norm(self.region.peers, self.N, self.rank, self.cap, self.H, [0] * 6, self.step_ctr,
                                 2 * self.n_layers, seq_layer, self.timeout_ns, self.status, self.off_recv[which],
                                 self.off_flag[which], x_res,
                                 next_norm if next_norm is not None else torch.empty(0, device=x_in.device),
                                 h_out, eps)
            ops.core._launched(2)
            return
        part = torch.zeros(T, W.N if hasattr(W, "N") else W.shape[0], dtype=torch.float32, device=x_in.device)
        ops.linear(x_in, W, part, ops.GEMV_ADD_F32)
        dist.all_reduce(part, group=self.ctx.group)
        x_res.add_(part)
        if next_norm is not None:
            ops.rms_norm(x_res, next_norm, eps, out=h_out)

    def part_view(self, rows: int) -> torch.Tensor:
        """f32 [rows, H] partial buffer of the two-shot all-reduce (rows <= prefill_rows)."""
        return self.region2.view(self.off_part, rows * self.H, torch.float32).view(rows, self.H)

    def twoshot_add(self, x_rows: torch.Tensor, next_norm=None, h_out=None, eps: float = 0.0):
        """x_rows += sum over ranks of their part_view(rows) (rank order; identical bits on every
        rank), then h_out = rmsnorm(x_rows) * next_norm when next_norm is given."""
        self.ts_seq += 1
        dev = x_rows.device
        ext().tp_twoshot(self.region2.peers, self.rank, self.off_part, self.off_gather, self.off_ready, self.off_done,
                         self.ts_seq, self.timeout_ns, self.status, self.ts_ctr, x_rows,
                         next_norm if next_norm is not None else torch.empty(0, device=dev),
                         h_out if h_out is not None else torch.empty(0, device=dev), eps)
        ops.core._launched(2)

    def allreduce_rows(self, T: int, partial_fn, x: torch.Tensor):
        """x[:T] += all_reduce(partial) in chunks of prefill_rows rows; partial_fn(r0, r1, out)
        writes this rank's f32 partial of rows [r0, r1) into out (a view of the region)."""
        for r0 in range(0, T, self.prefill_rows):
            r1 = min(T, r0 + self.prefill_rows)
            partial_fn(r0, r1, self.part_view(r1 - r0))
            self.twoshot_add(x[r0:r1])

    def check_status(self) -> int:
        return int(self.status.item()) if self.fused else 0


def shard_state(cfg, sd: dict, rank: int, size: int) -> dict:
    """Slices a canonical state dict for TP rank `rank` of `size`: attention by whole heads,
    dense FFNs by columns; in MoE layers every expert (and the shared expert) is split the same
    way along its FFN width (`TpSplit::experts`, reference crates/core/src/plan/stage.rs:103-109),
    the router stays whole."""
    hq, hk, d = cfg.n_heads // size, cfg.n_kv_heads // size, cfg.head_dim
    f = cfg.ffn // size
    fe = cfg.moe_ffn // size if cfg.n_experts else 0
    fs = fe * cfg.n_shared_experts if cfg.n_experts else 0
    out = {}
    for n, t in sd.items():
        leaf = n.split(".")[-1]
        if ".experts." in n or n.startswith("experts."):
            if leaf in ("gate", "up"):    # [E, f, h]
                out[n] = t[:, rank * fe:(rank + 1) * fe]
            elif leaf == "down":          # [E, h, f]
                out[n] = t[:, :, rank * fe:(rank + 1) * fe]
            else:
                out[n] = t
        elif ".shared." in n or n.startswith("shared."):
            if leaf in ("gate", "up"):
                out[n] = t[rank * fs:(rank + 1) * fs]
            elif leaf == "down":
                out[n] = t[:, rank * fs:(rank + 1) * fs]
            else:
                out[n] = t
        elif leaf in ("q_proj", "q_bias"):
            out[n] = t[rank * hq * d:(rank + 1) * hq * d]
        elif leaf in ("k_proj", "v_proj", "k_bias", "v_bias"):
            out[n] = t[rank * hk * d:(rank + 1) * hk * d]
        elif leaf == "o_proj":
            out[n] = t[:, rank * hq * d:(rank + 1) * hq * d]
        elif leaf in ("gate", "up"):
            out[n] = t[rank * f:(rank + 1) * f]
        elif leaf == "down":
            out[n] = t[:, rank * f:(rank + 1) * f]
        elif n == "lm_head" and cfg.vocab % size == 0 and (cfg.vocab // size) % 16 == 0:
            v = cfg.vocab // size  # vocab-parallel head: each rank scores its slice of the vocabulary
            out[n] = t[rank * v:(rank + 1) * v]
        else:
            out[n] = t
    return out


def local_config(cfg, size: int):
    assert cfg.n_heads % size == 0 and cfg.n_kv_heads % size == 0 and cfg.ffn % size == 0, \
        "heads, KV heads and FFN width must divide by the TP size"
    assert not cfg.is_mla, "tensor parallelism covers GQA attention (MLA models use expert parallelism)"
    kw = {}
    if cfg.n_experts:
        assert cfg.moe_ffn % (64 * size) == 0, "expert FFN width / TP size must be a multiple of 64"
        kw["moe_ffn"] = cfg.moe_ffn // size
    return cfg.replace(n_heads=cfg.n_heads // size, n_kv_heads=cfg.n_kv_heads // size, ffn=cfg.ffn // size, **kw)
