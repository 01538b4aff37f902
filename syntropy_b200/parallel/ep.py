"""Expert parallelism for the MoE FFN.

Each of N ranks owns E/N consecutive experts of every MoE layer and serves its own
sequences' attention (data-parallel attention).  Two data planes:

* fused (default on GPUs): router top-k -> ep_dispatch (P2P stores of rows into the
  owners' slots) -> ep_build (bounded waits, CSR of local experts) -> grouped GEMVs whose
  down-projection epilogue stores f32 rows straight into the source rank's combine
  buffer -> ep_combine (ascending-expert sum + next RMSNorm).  csrc/cuda/ep.cu.
* baseline (NCCL, any device): all-gather of every rank's rows, local experts applied to
  all rows, reduce-scatter of the f32 partial outputs.  This is the comparison baseline
  and the prefill path.

Reference design: plan/rfcs/RFC-0032-distributed-execution.md:415-424 (EP dispatch and
combine), crates/core/src/plan/stage.rs:54-130 (`ExpertOwnerMap`).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .._ext import ext
from .dist import DistContext
from .collectives import all_gather_rows, reduce_scatter_rows
from .symm import SymmetricRegion


def _align(n, a=256):
    return (n + a - 1) // a * a


class EPGroup:
    """Owns the symmetric region and per-step device state of expert parallelism."""

    def __init__(self, ctx: DistContext, n_experts: int, top_k: int, hidden: int, cap: int, n_layers: int,
                 timeout_s: float = 2.0, fused: bool = True):
        self.ctx = ctx
        self.N, self.rank = ctx.world, ctx.rank
        assert n_experts % self.N == 0, "experts must divide evenly over ranks"
        self.E, self.E_loc, self.k, self.H, self.cap = n_experts, n_experts // self.N, top_k, hidden, cap
        self.n_layers = n_layers
        self.fused = fused and ctx.device.type == "cuda"
        self.timeout_ns = int(timeout_s * 1e9)
        self.expert_range = (self.rank * self.E_loc, (self.rank + 1) * self.E_loc)
        if self.fused:
            N, cap, H, k = self.N, cap, hidden, top_k
            ms = 1 + 3 * k
            off = 0
            self.off_x = off
            off = _align(off + N * cap * H * 2)
            self.off_meta = off
            off = _align(off + N * cap * ms * 4)
            self.off_cnt = off
            off = _align(off + N * 4)
            self.off_flag_disp = off
            off = _align(off + N * 4)
            self.off_comb = off
            off = _align(off + cap * k * H * 4)
            self.off_flag_comb = off
            off = _align(off + N * 4)
            self.region = SymmetricRegion(ctx, off)
            self.offs = [self.off_x, self.off_meta, self.off_cnt, self.off_flag_disp, self.off_comb,
                         self.off_flag_comb]
            dev = ctx.device
            self.step_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.done_ctr = torch.zeros(n_layers, dtype=torch.int32, device=dev)
            self.collect_ctr = torch.zeros(1, dtype=torch.int32, device=dev)  # CPU-tier collect arrivals
            self._no_flags = torch.empty(0, dtype=torch.int32, device=dev)
            P = N * cap * k
            self.tok_off = torch.zeros(self.E_loc + 1, dtype=torch.int32, device=dev)
            self.tok_idx = torch.zeros(P, dtype=torch.int32, device=dev)
            self.pair_w = torch.zeros(P, dtype=torch.float32, device=dev)
            self.pair_dst = torch.zeros(P, dtype=torch.int64, device=dev)
            self.recv_x = self.region.view(self.off_x, N * cap * H, torch.bfloat16).view(N * cap, H)

    # ------------------------------------------------------------------ fused path
    def _common(self, layer):
        return (self.region.peers, self.N, self.rank, self.cap, self.H, self.k, self.E_loc, self.offs, self.step_ctr,
                self.n_layers, layer, self.timeout_ns, self.status)

    def step_begin(self):
        if self.fused:
            ext().ep_step_begin(self.step_ctr)

    def moe_decode_fused(self, layer: int, h, topk_ids, topk_w, x, gu, dn, mid, next_norm, h_out, eps,
                         stamp=None, tier=None, L=None, before_gemv=None, after_dispatch=None):
        """One MoE layer for the local rows (h: bf16 [T, H]) through NVLink dispatch/combine.
        stamp: device-timestamp callback of a profiled step; tier: the host CPU expert tier,
        which computes its share of this rank's cold experts for every rank's rows while the
        GPU runs the rest (its rows reach the sources' combine slots over NVLink); L: the
        model layer (its expert banks tell which experts the CPU owns); before_gemv: called right
        before the expert GEMVs (after dispatch and the CPU hand-off); after_dispatch: local work
        that overlaps the rows' flight to their owners (e.g. a shared expert adding into x).
        4-bit and block-scaled fp8 experts (gu.is_fp8): the fp8 path quantises the received rows
        and the SwiGLU rows to e4m3 (1x128 scales) before each GEMV; the down GEMV of both stores
        each pair's row into its source rank's combine slot and raises the layer's flags."""
        e = ext()
        c = self._common(layer)
        stamp = stamp or (lambda _lab: None)
        e.ep_dispatch(*c, h, topk_ids, topk_w)
        stamp(f"layer{layer}.dispatch")
        if after_dispatch is not None:
            after_dispatch()
        e.ep_build(*c, self.tok_off, self.tok_idx, self.pair_w, self.pair_dst)
        stamp(f"layer{layer}.build")
        # every layer hands off when a tier exists (the CPU answers with no rows for a layer whose
        # cold experts it does not own), so ownership changes between steps need no new capture
        cpu = tier is not None and L is not None and id(L) in tier.layer_of
        if cpu:
            tier.handoff_ep(tier.layer_of[id(L)], self.recv_x, self.tok_off, self.tok_idx, self.pair_w)
            ops.core._launched()
        P = self.N * self.cap * self.k
        if before_gemv is not None:  # e.g. wait for this layer's staged host experts
            before_gemv()
        ops.linear_grouped(self.recv_x, gu, self.tok_off, self.tok_idx, mid[:P], ops.GEMV_SWIGLU,
                           qw_ptrs=gu.qw_ptrs, sm_ptrs=gu.sm_ptrs)
        stamp(f"layer{layer}.gate_up")
        flags = self._no_flags if cpu else self.done_ctr[layer:layer + 1]
        nt = ops.moe_nt_hint(self.N * h.shape[0] * self.k // self.N, self.E_loc)
        if getattr(dn, "is_fp8", False):
            xq, xs = e.f8_quant_act(mid[:P])
            e.f8_gemv_ep(xq, xs, dn.qw_ptrs, dn.sm_ptrs, self.tok_off, self.pair_w, self.pair_dst, dn.N, dn.K, flags,
                         self.region.peers, self.off_flag_comb, self.rank, self.step_ctr, self.n_layers, layer, nt)
            ops.core._launched()
        else:
            e.q4_gemv_ep(mid[:P], dn.qw_ptrs, dn.sm_ptrs, self.tok_off,
                         torch.empty(0, dtype=torch.int32, device=h.device), self.pair_w, self.pair_dst, dn.N, dn.K,
                         flags, self.region.peers, self.off_flag_comb, self.rank, self.step_ctr, self.n_layers, layer,
                         nt, self.E_loc, bool(getattr(dn, "bank_contiguous", False)))
        stamp(f"layer{layer}.down")
        if cpu:  # the CPU's rows, then this layer's completion flags
            tier.collect_ep(self.pair_dst, layer)
            ops.core._launched()
            stamp(f"layer{layer}.cpu_wait")
        e.ep_combine(*c, x, next_norm if next_norm is not None else torch.empty(0, device=h.device), h_out, eps)
        stamp(f"layer{layer}.combine")
        ops.core._launched(5)

    def check_status(self) -> int:
        return int(self.status.item()) if self.fused else 0

    # ------------------------------------------------------------------ NCCL baseline
    def moe_baseline(self, h, topk_ids, topk_w, gu, dn, eps_unused=None, staged=None) -> torch.Tensor:
        """Returns f32 [T, H] MoE output for the local rows via all-gather + local experts +
        reduce-scatter.  Row counts are equalised by padding to the max over ranks."""
        ctx = self.ctx
        T = h.shape[0]
        t_all = [torch.zeros(1, dtype=torch.int64) for _ in range(self.N)]
        dist.all_gather(t_all, torch.tensor([T], dtype=torch.int64), group=ctx.cpu_group)
        Tm = max(int(t) for t in t_all)
        dev = h.device

        def pad(t, fill=0):
            if t.shape[0] == Tm:
                return t.contiguous()
            out = torch.full((Tm,) + tuple(t.shape[1:]), fill, dtype=t.dtype, device=dev)
            out[:T] = t
            return out

        hp, ip, wp = pad(h), pad(topk_ids, -1), pad(topk_w)
        H = self.H
        ga = torch.empty(self.N * Tm, H, dtype=h.dtype, device=dev)
        gi = torch.empty(self.N * Tm, self.k, dtype=ip.dtype, device=dev)
        gw = torch.empty(self.N * Tm, self.k, dtype=wp.dtype, device=dev)
        all_gather_rows(ga, hp, ctx.group)
        all_gather_rows(gi, ip, ctx.group)
        all_gather_rows(gw, wp, ctx.group)
        part = _local_experts_apply(ga, gi, gw, gu, dn, self.expert_range, staged)
        out = torch.empty(Tm, H, dtype=torch.float32, device=dev)
        reduce_scatter_rows(out, part, ctx.group)
        return out[:T]


def _local_experts_apply(rows, ids, w, gu, dn, erange, staged=None) -> torch.Tensor:
    """f32 [R, H]: sum over each row's experts that fall in erange (ascending expert order).
    staged: ((gu_qw_ptrs, gu_sm_ptrs), (dn_qw_ptrs, dn_sm_ptrs)) with every expert in VRAM
    (the expert cache's staging bank) for the prefill GEMMs."""
    R, H = rows.shape[0], dn.N
    dev = rows.device
    ea, eb = erange
    out = torch.zeros(R, H, dtype=torch.float32, device=dev)
    if R == 0:
        return out
    k = ids.shape[1]
    flat_ids = ids.reshape(-1).long()
    mine = (flat_ids >= ea) & (flat_ids < eb)
    sel = torch.nonzero(mine).squeeze(1)
    if sel.numel() == 0:
        return out
    e_loc = flat_ids[sel] - ea
    tok = sel // k
    key = e_loc * R + tok
    order = torch.argsort(key)
    sel, e_loc, tok = sel[order], e_loc[order], tok[order]
    counts = torch.bincount(e_loc, minlength=eb - ea)
    tok_off = torch.zeros(eb - ea + 1, dtype=torch.int32, device=dev)
    tok_off[1:] = torch.cumsum(counts, 0).int()
    pw = w.reshape(-1)[sel].float().contiguous()
    tok_idx = tok.int().contiguous()
    P = sel.numel()
    f = gu.N // 2
    bk = getattr(gu, "bank_contiguous", False)
    if rows.is_cuda and gu.qw is not None and P > 256 and gu.N % 128 == 0 and dn.N % 128 == 0 and \
            (bk or staged is not None):
        # prefill-sized: gather rows per expert, then grouped tcgen05 GEMMs
        (gq, gs), (dq, ds) = staged if staged is not None else ((gu.qw_ptrs, gu.sm_ptrs), (dn.qw_ptrs, dn.sm_ptrs))
        a_rows = rows.index_select(0, tok.long()).contiguous()
        mid = torch.empty(P, f, dtype=rows.dtype, device=dev)
        ops.gemm_grouped(a_rows, gq, gs, tok_off, gu.N, gu.K, 1, None, mid, eb - ea,
                         gu.qw if bk else None, gu.sm if bk else None)
        yp = torch.empty(P, H, dtype=torch.float32, device=dev)
        ops.gemm_grouped(mid, dq, ds, tok_off, dn.N, dn.K, 2, pw, yp, eb - ea,
                         dn.qw if bk else None, dn.sm if bk else None)
    elif rows.is_cuda and gu.qw is not None and int(counts.max()) <= 256:
        mid = torch.empty(P, f, dtype=rows.dtype, device=dev)
        ops.linear_grouped(rows, gu, tok_off, tok_idx, mid, ops.GEMV_SWIGLU, qw_ptrs=gu.qw_ptrs, sm_ptrs=gu.sm_ptrs)
        yp = torch.empty(P, H, dtype=torch.float32, device=dev)
        ops.linear_grouped(mid, dn, tok_off, None, yp, ops.GEMV_SCALED_F32, route_w=pw, qw_ptrs=dn.qw_ptrs,
                           sm_ptrs=dn.sm_ptrs)
    else:
        yp = torch.empty(P, H, dtype=torch.float32, device=dev)
        offl = tok_off.tolist()
        for el in range(eb - ea):
            a, b = offl[el], offl[el + 1]
            if a == b:
                continue
            r = rows[tok_idx[a:b].long()]
            wg, wd = gu.weight(el), dn.weight(el)
            mid = ops.swiglu_interleaved_ref(r.to(wg.dtype) @ wg.t()).to(wd.dtype)
            yp[a:b] = pw[a:b, None] * (mid @ wd.t()).float()
    # ascending expert order per row: pairs are sorted by expert, so a sequential
    # index_add over expert-sorted pairs keeps the per-row order fixed
    out.index_add_(0, tok.long(), yp) if not rows.is_cuda else _ordered_add(out, tok, yp, k)
    return out


def _ordered_add(out, tok, yp, k):
    """Deterministic per-row sum of pair rows (pairs already sorted by expert): gather the
    j-th pair of every row into its own pass so each row's additions happen in order."""
    R = out.shape[0]
    # rank of each pair within its row (pairs of a row appear in ascending expert order)
    order = torch.argsort(tok * (1 << 20) + torch.arange(tok.numel(), device=tok.device))
    tok_s = tok[order]
    first = torch.ones_like(tok_s, dtype=torch.bool)
    first[1:] = tok_s[1:] != tok_s[:-1]
    idx = torch.arange(tok_s.numel(), device=tok.device)
    start = torch.cummax(torch.where(first, idx, torch.zeros_like(idx)), 0).values
    j = idx - start
    for jj in range(int(j.max()) + 1 if j.numel() else 0):
        m = j == jj
        out[tok_s[m].long()] += yp[order[m]]
    return out
