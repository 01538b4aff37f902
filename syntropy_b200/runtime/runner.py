"""Model runner: static device buffers, the decode forward (captured in one CUDA graph per
batch bucket) and the eager prefill forward.

Step inputs travel as ONE packed step descriptor (int64 words) copied host->device per
step, mirroring the reference's StepDesc-first graph design (crates/kernels/include/
syntropy/step_desc.h; plan/rfcs/RFC-0040-kernel-providers-and-backends.md:425-461).
"""
from __future__ import annotations

import math

import torch

from .._ext import ext
import torch.nn.functional as F

from .. import ops
from ..formats.q4 import Q4Weight
from ..kv.paged import PagedKVCache
from ..models.transformer import ModelWeights
from ..obs.nvtx import nvtx_ranged

BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 192, 256)  # rows past 64: verify windows of drafts


def bucket_for(n: int, buckets=BUCKETS, cap: int | None = None) -> int:
    """Graph bucket for n rows: the smallest bucket that holds them, never above `cap` (the
    runner's row count, itself the last bucket when it is not one of BUCKETS)."""
    for b in buckets:
        if n <= b:
            return b if cap is None else min(b, max(cap, n))
    raise ValueError(f"batch {n} exceeds the largest bucket {buckets[-1]}")


class StepDesc:
    """Packed per-step inputs.  Fields (rows = max_batch):
    tokens, pos, ctx_len, top_k : int32-valued; slot, seed, stream, counter : int64;
    temperature, top_p : f32 (bit-cast); block_tables [rows, max_blocks] int32."""

    INT_FIELDS = ("tokens", "pos", "ctx_len", "top_k")
    LONG_FIELDS = ("slot", "seed", "stream", "counter")
    F_FIELDS = ("temperature", "top_p")

    def __init__(self, rows: int, max_blocks: int, device):
        self.rows, self.max_blocks = rows, max_blocks
        n_i32 = rows * (len(self.INT_FIELDS) + len(self.F_FIELDS)) + rows * max_blocks
        n_i32 += (-n_i32) % 2
        n_i64 = rows * len(self.LONG_FIELDS)
        self.nbytes = n_i32 * 4 + n_i64 * 8
        pin = device.type == "cuda"
        self.host = torch.zeros(self.nbytes, dtype=torch.uint8, pin_memory=pin)
        self.dev = torch.zeros(self.nbytes, dtype=torch.uint8, device=device)
        self.h, self.d = self._views(self.host), self._views(self.dev)

    def _views(self, buf):
        rows, mb = self.rows, self.max_blocks
        n_i32 = rows * (len(self.INT_FIELDS) + len(self.F_FIELDS)) + rows * mb
        n_i32 += (-n_i32) % 2
        i32 = buf[: n_i32 * 4].view(torch.int32)
        i64 = buf[n_i32 * 4:].view(torch.int64)
        v = {}
        o = 0
        for f in self.INT_FIELDS:
            v[f] = i32[o:o + rows]
            o += rows
        for f in self.F_FIELDS:
            v[f] = i32[o:o + rows].view(torch.float32)
            o += rows
        v["block_tables"] = i32[o:o + rows * mb].view(rows, mb)
        o = 0
        for f in self.LONG_FIELDS:
            v[f] = i64[o:o + rows]
            o += rows
        return v

    def upload(self):
        self.dev.copy_(self.host, non_blocking=True)


class ModelRunner:
    def __init__(self, mw: ModelWeights, max_batch: int = 64, max_seq_len: int = 4096, num_blocks: int | None = None,
                 kv_dtype=None, use_graphs: bool = True, kv_budget_bytes: int | None = None, ep=None, tp=None,
                 pp=None):
        cfg = mw.cfg
        self.pp = pp  # parallel.pp.PPGroup or None
        self.ep = ep  # parallel.ep.EPGroup or None
        self.expert_cache = None  # experts.cache.ExpertCache when a VRAM cap is set
        self._pf_stream = None    # side stream of the router-predicted expert prefetch
        self._pf_events = {}
        self.profile_next = False  # next decode step replays the timestamped graph variant
        self.profile_prefill_next = False  # next prefill pass records per-layer timestamps
        self._stamping = False
        self._stamp_n = 0
        self._stamp_labels: list[str] = []
        self._stamp_buf = None
        self.tp = tp  # parallel.tp.TPGroup or None
        self.mw, self.cfg = mw, cfg
        self.device = mw.device
        self.is_cuda = self.device.type == "cuda"
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.block_size = 16
        self.max_blocks = (max_seq_len + self.block_size - 1) // self.block_size
        kv_dtype = kv_dtype or (torch.bfloat16 if self.is_cuda else torch.float32)
        self.is_mla = cfg.is_mla
        kv_layers = len(mw.layers) + (cfg.n_mtp if mw.mtp is not None else 0)
        kv_heads, kv_dim = (1, cfg.kv_lora_rank + cfg.qk_rope_dim) if cfg.is_mla else (cfg.n_kv_heads, cfg.head_dim)
        if num_blocks is None:
            per = PagedKVCache.bytes_per_block(kv_layers, kv_heads, kv_dim, self.block_size,
                                               torch.tensor([], dtype=kv_dtype).element_size())
            if kv_budget_bytes is None:
                num_blocks = max_batch * self.max_blocks + 1
            else:
                num_blocks = max(2, kv_budget_bytes // per)
        self.kv = PagedKVCache(kv_layers, num_blocks, kv_heads, kv_dim, self.block_size, kv_dtype, self.device,
                               with_v=not cfg.is_mla)
        self.desc = StepDesc(max_batch, self.max_blocks, self.device)
        self.use_graphs = use_graphs and self.is_cuda
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.time_events: list | None = None  # when a list: (start, end) CUDA events per decode
        self._alloc_buffers()
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        # per-expert routed-pair counts of every layer, accumulated by the routing kernels
        # (captured graphs included) and folded into the expert cache's scores between steps
        self.route_counts = torch.zeros(len(mw.layers), cfg.n_experts, dtype=torch.int32, device=self.device) \
            if cfg.n_experts else None
        self._layer_index = {id(L): i for i, L in enumerate(mw.layers)}
        self.expert_stats = None
        self.expert_hit_rate = None  # VRAM hit rate of the last expert-cache rebalance window

    # ------------------------------------------------------------------ buffers
    def _alloc_buffers(self):
        cfg, B, dev = self.cfg, self.max_batch, self.device
        act = torch.bfloat16 if self.is_cuda else torch.float32
        H = cfg.hidden
        qkv_dim = cfg.q_dim + 2 * cfg.kv_dim
        b = {}
        b["x"] = torch.zeros(B, H, dtype=torch.float32, device=dev)
        b["h"] = torch.zeros(B, H, dtype=act, device=dev)
        if cfg.is_mla:
            b["attn"] = torch.zeros(B, cfg.n_heads, cfg.v_head_dim, dtype=act, device=dev)
        else:
            b["qkv"] = torch.zeros(B, qkv_dim, dtype=act, device=dev)
            b["q"] = torch.zeros(B, cfg.n_heads, cfg.head_dim, dtype=act, device=dev)
            b["attn"] = torch.zeros(B, cfg.n_heads, cfg.head_dim, dtype=act, device=dev)
        vl = self._vocab_local()
        if self._fused_head():
            # every rank's logits slice lands in this buffer (symmetric region) from the head GEMM
            b["logits"] = self.tp.logits_view(B)
        else:
            b["logits"] = torch.zeros(B, cfg.vocab, dtype=torch.float32, device=dev)
        if self.tp is not None and vl < cfg.vocab and not self._fused_head():  # local slice + gather space
            b["logits_local"] = torch.zeros(B, vl, dtype=torch.float32, device=dev)
            b["logits_gather"] = torch.zeros(self.tp.N * B, vl, dtype=torch.float32, device=dev)
        b["next"] = torch.zeros(B, dtype=torch.int32, device=dev)
        if any(not L.is_moe for L in self.mw.layers):
            b["ffn_mid"] = torch.zeros(B, cfg.ffn, dtype=act, device=dev)
        if cfg.is_moe:
            E, k = cfg.n_experts, cfg.top_k
            ep = self.ep
            if ep is not None and not ep.fused:  # NCCL all-gather / reduce-scatter rows
                B = B * ep.N  # baseline routes every rank's rows on every rank
                b["h_all"] = torch.zeros(B, H, dtype=act, device=dev)
                b["x_part"] = torch.zeros(B, H, dtype=torch.float32, device=dev)
                b["moe_red"] = torch.zeros(self.max_batch, H, dtype=torch.float32, device=dev)
            if self.tp is not None:  # experts split along their FFN width: partial MoE outputs
                b["tp_moe_part"] = torch.zeros(self.max_batch, H, dtype=torch.float32, device=dev)
            b["rlogits"] = torch.zeros(B, 2 * E, dtype=torch.float32, device=dev)
            b["topk_ids"] = torch.zeros(B, k, dtype=torch.int32, device=dev)
            b["topk_w"] = torch.zeros(B, k, dtype=torch.float32, device=dev)
            b["tok_off"] = torch.zeros(E + 1, dtype=torch.int32, device=dev)
            b["tok_idx"] = torch.zeros(B * k, dtype=torch.int32, device=dev)
            b["pair_w"] = torch.zeros(B * k, dtype=torch.float32, device=dev)
            b["pair_of"] = torch.zeros(B, k, dtype=torch.int32, device=dev)
            b["pred_mask"] = torch.zeros(E, dtype=torch.int32, device=dev)
            n_pairs = B * k
            if ep is not None and ep.fused:
                n_pairs = max(n_pairs, ep.N * ep.cap * k)
            b["moe_mid"] = torch.zeros(n_pairs, cfg.moe_ffn, dtype=act, device=dev)
            b["moe_out"] = torch.zeros(B * k, H, dtype=torch.float32, device=dev)
            B = self.max_batch
        # split-KV workspace sized for the largest split count
        self.pages_per_split = 16
        n_splits = (self.max_blocks + self.pages_per_split - 1) // self.pages_per_split
        if self.is_cuda and cfg.is_mla and cfg.kv_lora_rank == 512 and cfg.qk_rope_dim == 64 and cfg.n_heads % 16 == 0:
            # MLA decode kernel: enough KV splits for ~2 CTAs per SM at the largest batch
            per_split = B * (cfg.n_heads // 16)
            ns = max(1, min(self.max_blocks, -(-296 // per_split)))
            self.mla_pages_per_split = -(-self.max_blocks // ns)
            ns = -(-self.max_blocks // self.mla_pages_per_split)
            from ..models.reference import mla_softmax_scale
            self.mla_scale = mla_softmax_scale(cfg)
            b["mla_olat"] = torch.zeros(B, cfg.n_heads, 512, dtype=torch.float32, device=dev)
            b["mla_qcat"] = torch.zeros(B, cfg.n_heads, 512 + cfg.qk_rope_dim, dtype=torch.bfloat16, device=dev)
            b["mla_po"] = torch.zeros(B * cfg.n_heads * ns * 512, dtype=torch.float32, device=dev)
            b["mla_pml"] = torch.zeros(B * cfg.n_heads * ns * 2, dtype=torch.float32, device=dev)
        if self.is_cuda and not cfg.is_mla:
            b["part_o"] = torch.zeros(B * cfg.n_kv_heads * n_splits * 16 * cfg.head_dim, dtype=torch.float32,
                                      device=dev)
            b["part_ml"] = torch.zeros(B * cfg.n_kv_heads * n_splits * 16 * 2, dtype=torch.float32, device=dev)
        self.buf = b

    # ------------------------------------------------------------------ decode
    def _moe_bufs(self, B):
        b = self.buf
        k = self.cfg.top_k
        return {"topk_ids": b["topk_ids"][:B], "topk_w": b["topk_w"][:B], "tok_off": b["tok_off"],
                "tok_idx": b["tok_idx"][:B * k], "pair_w": b["pair_w"][:B * k], "pair_of": b["pair_of"][:B],
                "pred_mask": b["pred_mask"]}

    def decode_forward(self, B: int):
        """Forward of the first B rows of the step descriptor; writes logits and next tokens."""
        cfg, mw, b, d = self.cfg, self.mw, self.buf, self.desc.d
        x, h = b["x"][:B], b["h"][:B]
        if self._stamping:
            if self._stamp_buf is None:
                self._stamp_buf = torch.zeros(12 * len(mw.layers) + 8, dtype=torch.int64, device=self.device)
            self._stamp_n = 0
            self._stamp_labels = []
        self._stamp("start")
        if self.ep is not None:
            self.ep.step_begin()
        if self.tp is not None:
            self.tp.step_begin()
        self._stage_ev = {}
        cache = self.expert_cache
        if cache is not None and cache.stage_all:  # bulk staging of the first two MoE layers
            for li in range(min(2, len(cache.layers))):
                self._stage_issue(li)
        pp = self.pp
        if pp is None or pp.first:
            ops.embed(mw.embed, d["tokens"][:B], x)
        else:
            pp.recv_hidden(x)
        n_layers = len(mw.layers)
        first = mw.layers[0]
        ops.rms_norm(x, first.attn_norm, cfg.rms_eps, out=h)
        for i, L in enumerate(mw.layers):
            nxt = mw.layers[i + 1] if i + 1 < n_layers else None
            self._attention_decode(L, B, i)
            self._stamp(f"layer{i}.attention")
            if L.is_moe:
                self._moe_decode(L, nxt, B, i)
            else:
                nw = nxt.attn_norm if nxt else mw.final_norm
                if self.tp is None:
                    ops.rms_norm(x, L.ffn_norm, cfg.rms_eps, out=h)
                mid = b["ffn_mid"][:B]
                ops.linear(h, L.gate_up, mid, ops.GEMV_SWIGLU)
                if self.tp is not None:
                    self.tp.row_parallel_reduce(1, i, mid, L.down, x, nw, h, cfg.rms_eps)
                else:
                    ops.linear(mid, L.down, x, ops.GEMV_ADD_F32)
                    ops.rms_norm(x, nw, cfg.rms_eps, out=h)
            self._stamp(f"layer{i}.{'moe' if L.is_moe else 'ffn'}")
        logits = b["logits"][:B]
        if pp is not None and not pp.last:
            pp.send_hidden(x)
            pp.broadcast_tokens(b["next"][:B])
            return logits
        self._lm_head(h, logits, b.get("logits_local"), b.get("logits_gather"))
        self._stamp("lm_head")
        ops.sample(logits, d["temperature"][:B], d["top_k"][:B], d["top_p"][:B], d["seed"][:B], d["stream"][:B],
                   d["counter"][:B], b["next"][:B])
        self._stamp("sample")
        if pp is not None:
            pp.broadcast_tokens(b["next"][:B])
        return logits

    def _attention_decode_mla(self, L, B, i):
        """MLA decode for B rows (absorbed form over the paged latent cache)."""
        from ..models.mla import mla_attend, mla_qkv, mla_qkv_decode
        cfg, b, d = self.cfg, self.buf, self.desc.d
        h = b["h"][:B]
        pos = d["pos"][:B]
        out = b["attn"][:B].view(B, -1)
        if "mla_olat" in b and self.kv.k[i].dtype == torch.bfloat16:
            # projections, latent write and both absorbs in four kernels around the latent
            # attention (padding rows, slot -1, write the null page: capturable, no host sync)
            qcat = mla_qkv_decode(cfg, L.mla, h, pos, d["slot"][:B], self.mw.rope_cos, self.mw.rope_sin,
                                  self.kv.k[i], b["mla_qcat"][:B])
            o_lat = b["mla_olat"][:B]
            ops.mla_decode(qcat, self.kv.k[i], d["block_tables"][:B], d["ctx_len"][:B], o_lat, self.mla_scale,
                           b["mla_po"], b["mla_pml"], self.mla_pages_per_split)
            ext().mla_o_absorb(o_lat, L.mla["w_uv"], out)
            ops.core._launched()
            ops.linear(out, L.o, b["x"][:B], ops.GEMV_ADD_F32)
            return
        q_lat, q_pe, lat = mla_qkv(cfg, L.mla, h, pos, self.mw.rope_cos, self.mw.rope_sin)
        cache = self.kv.k[i].view(-1, self.kv.k[i].shape[-1])
        sl = d["slot"][:B].long()
        # padding rows (slot -1) write into the null page: no host sync, capturable
        cache.index_copy_(0, torch.where(sl >= 0, sl, torch.zeros_like(sl)), lat.to(cache.dtype))
        bs = self.block_size
        for r in range(B):
            n = int(d["ctx_len"][r])
            blocks = d["block_tables"][r, : (n + bs - 1) // bs]
            p_ = torch.arange(n, device=h.device)
            rows = cache[blocks[p_ // bs].long() * bs + p_ % bs]
            out[r] = mla_attend(cfg, L.mla, q_lat[r:r + 1], q_pe[r:r + 1], rows, 0)[0].to(out.dtype)
        ops.linear(out, L.o, b["x"][:B], ops.GEMV_ADD_F32)

    def _attention_decode(self, L, B, i):
        if self.is_mla:
            return self._attention_decode_mla(L, B, i)
        cfg, b, d = self.cfg, self.buf, self.desc.d
        h = b["h"][:B]
        qkv = b["qkv"][:B]
        ops.linear(h, L.qkv, qkv, ops.GEMV_STORE)
        if L.qkv_bias is not None:
            qkv.add_(L.qkv_bias)
        q = b["q"][:B]
        ops.qk_rope_kv_write(qkv, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, L.q_norm, L.k_norm, cfg.rms_eps,
                             d["pos"][:B], self.mw.rope_cos, self.mw.rope_sin, d["slot"][:B], q, self.kv.k[i],
                             self.kv.v[i])
        attn = b["attn"][:B]
        ops.attn_decode(q, self.kv.k[i], self.kv.v[i], d["block_tables"][:B], d["ctx_len"][:B], attn, self.scale,
                        b.get("part_o"), b.get("part_ml"), self.pages_per_split)
        if self.tp is not None:  # o_proj partials reduced over NVLink; h = ffn_norm(x)
            self.tp.row_parallel_reduce(0, i, attn.view(B, -1), L.o, b["x"][:B], L.ffn_norm, b["h"][:B], cfg.rms_eps)
        else:
            ops.linear(attn.view(B, -1), L.o, b["x"][:B], ops.GEMV_ADD_F32)

    def _moe_decode(self, L, nxt, B, layer):
        cfg, mw, b = self.cfg, self.mw, self.buf
        x, h = b["x"][:B], b["h"][:B]
        ops.rms_norm(x, L.ffn_norm, cfg.rms_eps, out=h)
        nw = nxt.attn_norm if nxt else mw.final_norm
        ep = self.ep
        if ep is not None and not ep.fused:
            return self._moe_decode_baseline(L, B, nw)
        pred = L.router_cat is not None
        rw = L.router_cat if pred else L.router
        E = cfg.n_experts
        W = 2 * E if pred else E
        rl = b["rlogits"].view(-1)[: B * W].view(B, W)
        ops.router_logits(h, rw, rl)
        mb = self._moe_bufs(B)
        cache = self.expert_cache
        nxt_moe = pred and cache is not None and cache.prefetch and layer + 1 < len(mw.layers)
        if nxt_moe:  # the next layer's prediction goes to its own mask (read by the side stream)
            mb["pred_mask"] = mw.layers[layer + 1].expert_tier.pred
        # padding rows of the bucket (slot -1) route too, but are not counted
        ops.moe_topk(rl, cfg, L.router_bias, pred, mb, counts=self._counts_of(layer),
                     count_rows=self.desc.d["slot"][:B])
        self._stamp(f"layer{layer}.route")
        if nxt_moe:
            # router-predicted prefetch of layer+1's host experts, overlapping this layer
            cur = torch.cuda.current_stream(self.device)
            if self._pf_stream is None:
                self._pf_stream = torch.cuda.Stream(device=self.device)
            self._pf_stream.wait_stream(cur)
            with torch.cuda.stream(self._pf_stream):
                cache.decode_prefetch(mw.layers[layer + 1])
                ops.core._launched()
            ev = torch.cuda.Event()
            ev.record(self._pf_stream)
            self._pf_events[layer + 1] = ev
        ev = self._pf_events.pop(layer, None)
        if ev is not None:  # this layer's pointer tables and staged experts are ready
            torch.cuda.current_stream(self.device).wait_event(ev)
        li = self._cache_index(L) if cache is not None and cache.stage_all else None

        def staged():
            # the GPU-read host experts of this layer are in its staging bank (waited for only
            # right before the GEMVs that read them: routing and the CPU hand-off go first)
            ev = self._stage_ev.pop(li, None) if li is not None else None
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
        k = cfg.top_k
        gu, dn = L.experts_gu, L.experts_down
        if ep is not None:
            # the shared expert (every rank holds it whole) adds into x while the rows fly to their owners
            shared_into_x = (lambda: self._shared_expert(L, h, into=x)) if L.shared_gu is not None else None
            ep.moe_decode_fused(layer, h, mb["topk_ids"], mb["topk_w"], x, gu, dn, b["moe_mid"], nw, h,
                                cfg.rms_eps, stamp=self._stamp if self._stamping else None,
                                tier=cache.cpu_tier if cache is not None else None, L=L, before_gemv=staged,
                                after_dispatch=shared_into_x)
            if li is not None:  # this layer's staging bank is free: stage the layer after next
                self._stage_issue(li + 2)
            return
        mid = b["moe_mid"][:B * k]
        yp = b["moe_out"][:B * k]
        tier = cache.cpu_tier if cache is not None else None
        if tier is not None:  # the host CPU computes its share of the cold experts meanwhile
            tier.handoff(L, h, mb)
            ops.core._launched()
        shared = self._shared_expert(L, h) if L.shared_gu is not None else None
        staged()
        ops.linear_grouped(h, gu, mb["tok_off"], mb["tok_idx"], mid, ops.GEMV_SWIGLU,
                           qw_ptrs=gu.qw_ptrs, sm_ptrs=gu.sm_ptrs)
        self._stamp(f"layer{layer}.gate_up")
        ops.linear_grouped(mid, dn, mb["tok_off"], None, yp, ops.GEMV_SCALED_F32, route_w=mb["pair_w"],
                           qw_ptrs=dn.qw_ptrs, sm_ptrs=dn.sm_ptrs)
        self._stamp(f"layer{layer}.down")
        if li is not None:  # this layer's staging bank is free: stage the layer after next
            self._stage_issue(li + 2)
        if tier is not None:
            tier.collect(yp)
            ops.core._launched()
            self._stamp(f"layer{layer}.cpu_wait")
        if self.tp is not None:
            # every expert holds 1/N of its FFN width here: combine the partial outputs, sum them
            # over the TP group (NCCL, captured in the decode graphs), then residual + next norm
            import torch.distributed as dist
            part = b["tp_moe_part"][:B]
            part.zero_()
            ops.moe_combine_rmsnorm(part, yp, mb["pair_of"], shared, None, None, cfg.rms_eps)
            dist.all_reduce(part, group=self.tp.ctx.group)
            x.add_(part)
            ops.rms_norm(x, nw, cfg.rms_eps, out=h)
            return
        ops.moe_combine_rmsnorm(x, yp, mb["pair_of"], shared, nw, h, cfg.rms_eps)

    def _cache_index(self, L):
        idx = getattr(self, "_cache_idx", None)
        if idx is None:
            idx = self._cache_idx = {id(X): i for i, X in enumerate(self.expert_cache.layers)}
        return idx.get(id(L))

    def _stage_issue(self, li: int):
        """Bulk staging copy of MoE layer li (cache order) on the side stream, after everything
        enqueued so far on the compute stream (which includes the last reader of its bank)."""
        cache = self.expert_cache
        if li >= len(cache.layers):
            return
        cur = torch.cuda.current_stream(self.device)
        if self._pf_stream is None:
            self._pf_stream = torch.cuda.Stream(device=self.device)
        self._pf_stream.wait_stream(cur)
        with torch.cuda.stream(self._pf_stream):
            cache.issue_stage_copy(li)
        ev = torch.cuda.Event()
        ev.record(self._pf_stream)
        self._stage_ev[li] = ev

    def after_step(self):
        """Host-side checks after a decode step has been synchronised (device status words of
        the CPU expert hand-off)."""
        tier = self.expert_cache.cpu_tier if self.expert_cache is not None else None
        if tier is not None:
            tier.check()

    def _counts_of(self, layer: int):
        return self.route_counts[layer] if self.route_counts is not None and self.expert_cache is not None else None

    def _counts_for(self, L):
        i = self._layer_index.get(id(L))  # the MTP block's layer is not a cached layer
        return self._counts_of(i) if i is not None else None

    def adapt_experts(self, max_swaps_per_layer: int = 2) -> int:
        """Expert-cache adaptation between steps: fold the routing counts accumulated since
        the last call into the decayed-LFU scores and swap cold residents for hot host
        experts.  Pointer tables change in place, so captured decode graphs stay valid.
        Under expert parallelism the counts are summed over the group first (every rank must
        call this at the same step).  Reference: crates/tier/src/experts/stats.rs:35-205."""
        cache = self.expert_cache
        if cache is None or self.route_counts is None:
            return 0
        from ..experts.cache import ExpertStats
        if self.expert_stats is None:
            self.expert_stats = ExpertStats(len(cache.layers), self.cfg.n_experts)
        c = self.route_counts
        if self.ep is not None:
            import torch.distributed as dist
            dist.all_reduce(c, group=self.ep.ctx.group)
        host = c.to("cpu", copy=True)  # a copy also on CPU runners: the counters are zeroed next
        c.zero_()
        hits = total = 0
        for li, L in enumerate(cache.layers):
            cnt = host[self._layer_index[id(L)]]
            self.expert_stats.observe(li, cnt)
            b = getattr(L, "expert_tier", None)
            if b is not None:
                resident = b.resident_mask()  # this rank's experts e0 .. e0 + E
                mine = cnt[b.e0: b.e0 + b.E]
                hits += int(mine[resident].sum())
                total += int(mine.sum())
        # share of the window's routed pairs whose expert was in VRAM (before this rebalance)
        self.expert_hit_rate = hits / total if total else None
        return cache.rebalance(self.expert_stats, max_swaps_per_layer)

    def _shared_expert(self, L, h, into=None):
        """Shared-expert FFN output (f32 [T, H]) added to the routed combine; with `into` (f32
        [T, H]) the output is added to that tensor instead."""
        T = h.shape[0]
        mid = torch.empty(T, L.shared_gu.N // 2 if hasattr(L.shared_gu, "N") else L.shared_gu.shape[0] // 2,
                          dtype=h.dtype, device=h.device)
        ops.linear(h, L.shared_gu, mid, ops.GEMV_SWIGLU)
        out = into if into is not None else torch.zeros(T, self.cfg.hidden, dtype=torch.float32, device=h.device)
        ops.linear(mid, L.shared_down, out, ops.GEMV_ADD_F32)
        return out

    def _moe_decode_baseline(self, L, B, nw):
        """NCCL baseline: all-gather rows, route all rows, apply local experts, reduce-scatter."""
        from ..parallel.collectives import all_gather_rows, reduce_scatter_rows
        cfg, b, ep = self.cfg, self.buf, self.ep
        N, k, E = ep.N, cfg.top_k, cfg.n_experts
        x, h = b["x"][:B], b["h"][:B]
        ha = b["h_all"][: N * B]
        all_gather_rows(ha, h, ep.ctx.group)
        R = N * B
        rl = b["rlogits"].view(-1)[: R * E].view(R, E)
        ops.router_logits(ha, L.router, rl)
        mb = self._moe_bufs(R)
        # every rank routes all rows here: rank 0 alone counts them (sums over the group later)
        ops.moe_topk(rl, cfg, L.router_bias, False, mb,
                     counts=self._counts_for(L) if ep.rank == 0 else None)
        ea, eb = ep.expert_range
        gu, dn = L.experts_gu, L.experts_down
        mid = b["moe_mid"][: R * k]
        yp = b["moe_out"][: R * k]
        yp.zero_()
        off = mb["tok_off"][ea: eb + 1]
        cache = self.expert_cache
        li = self._cache_index(L) if cache is not None and cache.stage_all else None
        ev = self._stage_ev.pop(li, None) if li is not None else None
        if ev is not None:  # the GPU-read host experts of this layer are in its staging bank
            torch.cuda.current_stream(self.device).wait_event(ev)
        ops.linear_grouped(ha, gu, off, mb["tok_idx"], mid, ops.GEMV_SWIGLU, qw_ptrs=gu.qw_ptrs, sm_ptrs=gu.sm_ptrs)
        ops.linear_grouped(mid, dn, off, None, yp, ops.GEMV_SCALED_F32, route_w=mb["pair_w"],
                           qw_ptrs=dn.qw_ptrs, sm_ptrs=dn.sm_ptrs)
        if li is not None:  # this layer's staging bank is free: stage the layer after next
            self._stage_issue(li + 2)
        part = b["x_part"][:R]
        part.zero_()
        ops.moe_combine_rmsnorm(part, yp, mb["pair_of"], None, None, None, cfg.rms_eps)
        red = b["moe_red"][:B]
        reduce_scatter_rows(red, part, ep.ctx.group)
        x.add_(red)
        if L.shared_gu is not None:  # every rank holds the shared expert whole: local rows only
            self._shared_expert(L, h, into=x)
        ops.rms_norm(x, nw, cfg.rms_eps, out=h)

    @nvtx_ranged("syn.decode")
    def decode(self, B: int):
        """Run one decode step for the first B rows (descriptor already filled on the host).
        With `profile_next` set, this step replays the profiled graph variant, which also
        writes device timestamps at every layer boundary (see `step_profile`)."""
        prof = self.profile_next and self.is_cuda
        self.profile_next = False
        self._stamping = prof
        if self.use_graphs:
            bb = bucket_for(B, cap=self.max_batch)
            key = ("profiled", bb) if prof else bb
            g = self.graphs.get(key)
            if g is None:
                g = self.capture(bb, key)  # uses (and restores) the host descriptor
            ev = self._ev0()
            # native: descriptor upload + graph launch on the current stream
            ext().step_launch(self.desc.host, self.desc.dev, g.raw_cuda_graph_exec(),
                              torch.cuda.current_stream(self.device).cuda_stream)
            self._ev1(ev)
        else:
            self.desc.upload()
            ev = self._ev0()
            self.decode_forward(B)
            self._ev1(ev)
        self._stamping = False
        return self.buf["next"][:B]

    # ------------------------------------------------------------------ output head
    def _vocab_local(self) -> int:
        W = self.mw.lm_head
        return int(getattr(W, "N", None) or W.shape[0])

    def _fused_head(self) -> bool:
        """Vocab-parallel bf16 head whose GEMM writes every rank's logits buffer (no NCCL)."""
        tp, W = self.tp, self.mw.lm_head
        return bool(tp is not None and getattr(tp, "vocab", 0) and isinstance(W, torch.Tensor) and
                    W.dtype == torch.bfloat16 and self._vocab_local() * tp.N == self.cfg.vocab and
                    self._vocab_local() % 32 == 0 and tp.cap >= self.max_batch)

    def _lm_head(self, h, logits, local=None, gathered=None):
        """logits [T, V] f32.  Under TP with a vocab-parallel head each rank scores its vocab
        slice and the slices are all-gathered in rank order (every rank then samples alike):
        fused into the head GEMM's epilogue over NVLink for bf16 heads, NCCL otherwise."""
        vl = self._vocab_local()
        if vl == self.cfg.vocab or self.tp is None:
            ops.linear(h, self.mw.lm_head, logits, ops.GEMV_STORE)
            return logits
        if self._fused_head() and logits.data_ptr() == self.buf["logits"].data_ptr():
            self.tp.gather_logits(h, self.mw.lm_head, h.shape[0])
            return logits
        from ..parallel.tp import gather_vocab_logits
        T = h.shape[0]
        if local is None:
            local = torch.empty(T, vl, dtype=torch.float32, device=h.device)
            gathered = torch.empty(self.tp.N * T, vl, dtype=torch.float32, device=h.device)
        local = local[:T]
        ops.linear(h, self.mw.lm_head, local, ops.GEMV_STORE)
        gather_vocab_logits(local, logits, gathered, self.tp.ctx.group)
        return logits

    # ------------------------------------------------------------------ profiled steps
    def _stamp(self, label: str):
        """Device timestamp at a segment boundary (profiled steps only; captured in the
        profiled graph variant)."""
        if not self._stamping:
            return
        n = self._stamp_n
        if self._stamp_buf is None or n >= self._stamp_buf.numel():
            return
        ops.timestamp(self._stamp_buf, n)
        if len(self._stamp_labels) <= n:
            self._stamp_labels.append(label)
        self._stamp_n = n + 1

    def step_profile(self) -> list[tuple[str, float]]:
        """Per-segment device time (ms) of the last profiled step: (segment label, ms)."""
        torch.cuda.synchronize(self.device)
        t = self._stamp_buf[: len(self._stamp_labels)].cpu().tolist()
        return [(self._stamp_labels[i], (t[i] - t[i - 1]) / 1e6) for i in range(1, len(t))]

    def _ev0(self):
        if self.time_events is None or not self.is_cuda:
            return None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        return (e0, e1)

    def _ev1(self, ev):
        if ev is not None:
            ev[1].record()
            self.time_events.append(ev)

    def capture(self, bb: int, key=None) -> "torch.cuda.CUDAGraph":
        """Capture the decode forward for bucket size bb (rows beyond the live batch are
        padding: null page, slot -1, greedy)."""
        d = self.desc.h
        saved = {k: v.clone() for k, v in d.items()}
        d["tokens"][:bb] = 0
        d["pos"][:bb] = 0
        d["ctx_len"][:bb] = 1
        d["slot"][:bb] = -1
        d["block_tables"][:bb] = 0
        d["temperature"][:bb] = 0
        d["top_k"][:bb] = 0
        d["top_p"][:bb] = 1
        self.desc.upload()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.decode_forward(bb)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.decode_forward(bb)
        torch.cuda.synchronize()
        for k, v in saved.items():
            d[k].copy_(v)
        self.graphs[bb if key is None else key] = g
        return g

    # ------------------------------------------------------------------ prefill
    pp_prefill_groups = 2  # pipeline parallelism: sequence groups handed between stages per prefill

    @torch.no_grad()
    @nvtx_ranged("syn.prefill")
    def prefill(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, cu_seqlens: list[int],
                prefix: list | None = None, block_lists: list | None = None):
        """Eager prefill of freshly started sequences (or of chunks after a cached prefix).
        block_lists: each sequence's KV pages (the paged attention kernel reads keys through
        them).  Returns the last-token logits of each sequence [n_seq, vocab] (f32).

        Under pipeline parallelism with several sequences the prefill is pipelined
        (reference RFC-0001 :1832-1899, chunked staggered prefill): the sequences form groups,
        each stage computes group k while the hidden states of group k-1 are still in flight
        to the next stage (asynchronous NCCL point-to-point), and the next stage has posted
        its receive of group k+1 before it computes group k."""
        pp = self.pp
        n = len(cu_seqlens) - 1
        G = min(self.pp_prefill_groups, n) if pp is not None else 1
        if G <= 1:
            return self._prefill_pass(tokens, positions, slots, cu_seqlens, prefix, block_lists)
        # contiguous sequence groups of about equal token counts
        bounds, total, acc = [0], cu_seqlens[-1], 0
        for s_i in range(n):
            acc = cu_seqlens[s_i + 1]
            if len(bounds) < G and acc >= total * len(bounds) / G and s_i + 1 < n:
                bounds.append(s_i + 1)
        bounds.append(n)
        groups = [(a, b) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
        dev = self.device

        def recv(g):
            a, b = groups[g]
            buf = torch.empty(cu_seqlens[b] - cu_seqlens[a], self.cfg.hidden, dtype=torch.float32, device=dev)
            return buf, pp.irecv_hidden(buf)

        pending = recv(0) if not pp.first else None
        sends, outs = [], []
        for g, (a, b) in enumerate(groups):
            nxt = recv(g + 1) if not pp.first and g + 1 < len(groups) else None
            x_in = None
            if pending is not None:
                x_in, work = pending
                work.wait()
            t0, t1 = cu_seqlens[a], cu_seqlens[b]
            res = self._prefill_pass(tokens[t0:t1], positions[t0:t1], slots[t0:t1], [c - t0 for c in cu_seqlens[a:b + 1]],
                                     prefix[a:b] if prefix is not None else None,
                                     block_lists[a:b] if block_lists is not None else None, x_in=x_in, pp_io=False)
            if pp.last:
                outs.append(res)
            else:
                sends.append((res, pp.isend_hidden(res)))
            pending = nxt
        for _, work in sends:
            work.wait()
        return torch.cat(outs, 0) if pp.last else None

    @torch.no_grad()
    def _prefill_pass(self, *args, **kw):
        """One prefill pass (see `_prefill_pass_body`); with `profile_prefill_next` set, the pass
        records device timestamps after each layer's attention and FFN (`step_profile`)."""
        prof = self.profile_prefill_next and self.is_cuda
        try:
            return self._prefill_pass_body(*args, **kw)
        finally:
            if prof:
                self._stamp("prefill_head")
                self._stamping = False

    def _prefill_pass_body(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                           cu_seqlens: list[int], prefix: list | None = None, block_lists: list | None = None,
                           x_in=None, pp_io: bool = True):
        """One prefill pass of this stage's layers.  pp_io: receive / send the hidden states
        here (blocking); otherwise x_in is the received input and the hidden states are
        returned instead of sent (pipelined prefill)."""
        cfg, mw, dev = self.cfg, self.mw, self.device
        T = tokens.numel()
        act = torch.bfloat16 if self.is_cuda else torch.float32
        prof = self.profile_prefill_next and self.is_cuda
        if prof:  # device timestamps around each layer's attention and FFN (eager pass)
            self.profile_prefill_next = False
            self._stamping = True
            if self._stamp_buf is None:
                self._stamp_buf = torch.zeros(12 * len(mw.layers) + 8, dtype=torch.int64, device=self.device)
            self._stamp_n = 0
            self._stamp_labels = []
            self._stamp("start")
        tokens = tokens.to(dev, torch.int32)
        positions = positions.to(dev, torch.int32)
        slots = slots.to(dev, torch.int64)
        pp = self.pp
        if x_in is not None:
            x = x_in
        else:
            x = torch.empty(T, cfg.hidden, dtype=torch.float32, device=dev)
            if pp is None or pp.first:
                ops.embed(mw.embed, tokens, x)
            else:
                pp.recv_hidden(x)
        h = torch.empty(T, cfg.hidden, dtype=act, device=dev)
        if not self.is_mla:
            qkv = torch.empty(T, cfg.q_dim + 2 * cfg.kv_dim, dtype=act, device=dev)
            q = torch.empty(T, cfg.n_heads, cfg.head_dim, dtype=act, device=dev)
            attn = torch.empty(T, cfg.n_heads, cfg.head_dim, dtype=act, device=dev)
        self._prefill_x = x
        paged = None
        if block_lists is not None and self.is_cuda and not self.is_mla and cfg.head_dim == 128 and T > 0:
            nseq = len(block_lists)
            width = max(1, max(len(b) for b in block_lists))
            bt = torch.zeros(nseq, width, dtype=torch.int32)
            for r, blocks in enumerate(block_lists):
                bt[r, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
            starts = [p[1] for p in prefix] if prefix is not None else [0] * nseq
            q_lens = [cu_seqlens[r + 1] - cu_seqlens[r] for r in range(nseq)]
            paged = (bt.to(dev), torch.tensor(cu_seqlens, dtype=torch.int32).to(dev),
                     torch.tensor([st + n for st, n in zip(starts, q_lens)], dtype=torch.int32).to(dev), max(q_lens))
        for i, L in enumerate(mw.layers):
            ops.rms_norm(x, L.attn_norm, cfg.rms_eps, out=h)
            if self.is_mla:
                self._prefill_mla(L, i, h, x, positions, slots, cu_seqlens, prefix)
                self._stamp(f"layer{i}.prefill_attn")
                ops.rms_norm(x, L.ffn_norm, cfg.rms_eps, out=h)
                if L.is_moe:
                    self._moe_prefill(L, h, x)
                else:
                    mid = torch.empty(T, cfg.ffn, dtype=act, device=dev)
                    ops.linear(h, L.gate_up, mid, ops.GEMV_SWIGLU)
                    self._row_parallel(mid, L.down, x)
                self._stamp(f"layer{i}.prefill_{'moe' if L.is_moe else 'ffn'}")
                continue
            ops.linear(h, L.qkv, qkv, ops.GEMV_STORE)
            if L.qkv_bias is not None:
                qkv.add_(L.qkv_bias)
            ops.qk_rope_kv_write(qkv, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, L.q_norm, L.k_norm, cfg.rms_eps,
                                 positions, mw.rope_cos, mw.rope_sin, slots, q, self.kv.k[i], self.kv.v[i])
            self._stamp(f"layer{i}.prefill_qkv")
            if paged is not None:
                ops.attn_prefill_paged(q, self.kv.k[i], self.kv.v[i], paged[0], paged[1], paged[2], attn, paged[3],
                                       self.scale)
            elif prefix is None or not any(p[1] for p in prefix):
                kc = self.kv.k[i].permute(0, 2, 1, 3).reshape(-1, cfg.n_kv_heads, cfg.head_dim)[slots]
                vc = self.kv.v[i].permute(0, 2, 1, 3).reshape(-1, cfg.n_kv_heads, cfg.head_dim)[slots]
                ops.attn_prefill(q, kc, vc, cu_seqlens, attn, self.scale)
            else:
                self._prefill_attn_with_prefix(i, q, attn, cu_seqlens, prefix)
            self._stamp(f"layer{i}.prefill_attn_core")
            self._row_parallel(attn.view(T, -1), L.o, x)
            self._stamp(f"layer{i}.prefill_attn")
            ops.rms_norm(x, L.ffn_norm, cfg.rms_eps, out=h)
            if L.is_moe:
                self._moe_prefill(L, h, x)
            else:
                mid = torch.empty(T, cfg.ffn, dtype=act, device=dev)
                ops.linear(h, L.gate_up, mid, ops.GEMV_SWIGLU)
                self._row_parallel(mid, L.down, x)
            self._stamp(f"layer{i}.prefill_{'moe' if L.is_moe else 'ffn'}")
        if len(cu_seqlens) == 1:
            return torch.zeros(0, cfg.vocab, dtype=torch.float32, device=dev)
        if pp is not None and not pp.last:
            if not pp_io:
                return x  # the pipelined caller sends it
            pp.send_hidden(x)
            return None  # the last stage produces the logits; tokens arrive by broadcast
        last = torch.tensor([c - 1 for c in cu_seqlens[1:]], device=dev, dtype=torch.long)
        hl = ops.rms_norm(x[last].contiguous(), mw.final_norm, cfg.rms_eps)
        logits = torch.empty(last.numel(), cfg.vocab, dtype=torch.float32, device=dev)
        self._lm_head(hl, logits)
        return logits

    def _prefill_mla(self, L, i, h, x, positions, slots, cu_seqlens, prefix):
        from ..models.mla import mla_attend, mla_qkv
        cfg = self.cfg
        q_lat, q_pe, lat = mla_qkv(cfg, L.mla, h, positions, self.mw.rope_cos, self.mw.rope_sin)
        cache = self.kv.k[i].view(-1, self.kv.k[i].shape[-1])
        ok = slots >= 0
        cache[slots[ok].long()] = lat[ok].to(cache.dtype)
        T = h.shape[0]
        out = torch.empty(T, cfg.n_heads * cfg.v_head_dim, dtype=h.dtype, device=h.device)
        bs = self.block_size
        for s_idx in range(len(cu_seqlens) - 1):
            a, b = cu_seqlens[s_idx], cu_seqlens[s_idx + 1]
            start = prefix[s_idx][1] if prefix else 0
            if start:
                blocks = torch.tensor(prefix[s_idx][0], device=h.device)
                p_ = torch.arange(start + b - a, device=h.device)
                rows = cache[blocks[p_ // bs].long() * bs + p_ % bs]
            else:
                rows = cache[slots[a:b].long()]
            out[a:b] = mla_attend(cfg, L.mla, q_lat[a:b], q_pe[a:b], rows, 0, causal_from=start).to(out.dtype)
        self._row_parallel(out, L.o, x)

    # ------------------------------------------------------------------ MTP drafting
    @torch.no_grad()
    def mtp_forward(self, x_prev: torch.Tensor, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                    block_tables: list) -> torch.Tensor:
        """One MTP-head step for S rows: from the main model's final residual at position j-1
        and the token at position j, write the MTP block's latent KV at j and return the
        argmax draft for position j+1."""
        from ..models.mla import mla_attend, mla_qkv
        cfg, mw, m = self.cfg, self.mw, self.mw.mtp
        dev = self.device
        S = x_prev.shape[0]
        act = torch.bfloat16 if self.is_cuda else torch.float32
        e = torch.empty(S, cfg.hidden, dtype=torch.float32, device=dev)
        ops.embed(mw.embed, tokens.to(dev, torch.int32), e)
        en = ops.rms_norm(e, m["enorm"], cfg.rms_eps)
        hn = ops.rms_norm(x_prev.to(dev), m["hnorm"], cfg.rms_eps)
        cat = torch.cat([en.to(act), hn.to(act)], -1).contiguous()
        x = torch.zeros(S, cfg.hidden, dtype=torch.float32, device=dev)
        ops.linear(cat, m["proj"], x, ops.GEMV_ADD_F32)
        L = m["block"]
        li = cfg.n_layers  # the MTP block's cache layer
        h = ops.rms_norm(x, L.attn_norm, cfg.rms_eps).to(act)
        pos = positions.to(dev)
        q_lat, q_pe, lat = mla_qkv(cfg, L.mla, h, pos, mw.rope_cos, mw.rope_sin)
        cache = self.kv.k[li].view(-1, self.kv.k[li].shape[-1])
        sl = slots.to(dev)
        cache[sl.long()] = lat.to(cache.dtype)
        out = torch.empty(S, cfg.n_heads * cfg.v_head_dim, dtype=act, device=dev)
        bs = self.block_size
        if "mla_olat" in self.buf and S <= self.max_batch:
            # decode-sized draft pass: the MLA decode kernel over the MTP block's latent cache
            width = self.desc.h["block_tables"].shape[1]
            bt = torch.zeros(S, width, dtype=torch.int32)
            for r in range(S):
                blk = block_tables[r][:width]
                bt[r, :len(blk)] = torch.tensor(blk, dtype=torch.int32)
            ctx = (positions.to(torch.int32) + 1)
            qcat = torch.cat([q_lat, q_pe], -1).to(torch.bfloat16).contiguous()
            o_lat = self.buf["mla_olat"][:S]
            ops.mla_decode(qcat, self.kv.k[li], bt.to(dev), ctx.to(dev), o_lat, self.mla_scale, self.buf["mla_po"],
                           self.buf["mla_pml"], self.mla_pages_per_split)
            ext().mla_o_absorb(o_lat, L.mla["w_uv"], out)
            ops.core._launched()
        else:
            for r in range(S):
                n = int(positions[r]) + 1
                blocks = torch.tensor(block_tables[r][: (n + bs - 1) // bs], device=dev)
                p_ = torch.arange(n, device=dev)
                rows = cache[blocks[p_ // bs].long() * bs + p_ % bs]
                out[r] = mla_attend(cfg, L.mla, q_lat[r:r + 1], q_pe[r:r + 1], rows, 0)[0].to(act)
        ops.linear(out, L.o, x, ops.GEMV_ADD_F32)
        h = ops.rms_norm(x, L.ffn_norm, cfg.rms_eps).to(act)
        if L.is_moe:
            self._moe_prefill(L, h.contiguous(), x)
        else:
            mid = torch.empty(S, cfg.ffn, dtype=act, device=dev)
            ops.linear(h, L.gate_up, mid, ops.GEMV_SWIGLU)
            ops.linear(mid, L.down, x, ops.GEMV_ADD_F32)
        hl = ops.rms_norm(x, mw.final_norm, cfg.rms_eps).to(act)
        logits = torch.empty(S, cfg.vocab, dtype=torch.float32, device=dev)
        self._lm_head(hl.contiguous(), logits)
        return torch.argmax(logits, -1).to(torch.int32).cpu()

    def _prefill_attn_with_prefix(self, i, q, attn, cu_seqlens, prefix):
        """Prefill attention for chunks that continue a cached prefix: queries are the new
        tokens, keys/values are every position of the sequence read from its pages."""
        import torch.nn.functional as F
        cfg = self.cfg
        kflat = self.kv.k[i].permute(0, 2, 1, 3).reshape(-1, cfg.n_kv_heads, cfg.head_dim)
        vflat = self.kv.v[i].permute(0, 2, 1, 3).reshape(-1, cfg.n_kv_heads, cfg.head_dim)
        for s_idx, (blocks, start) in enumerate(prefix):
            a, b = cu_seqlens[s_idx], cu_seqlens[s_idx + 1]
            n_new = b - a
            total = start + n_new
            pos = torch.arange(total, device=q.device)
            bt = torch.tensor(blocks, device=q.device, dtype=torch.long)
            sl = bt[pos // self.block_size] * self.block_size + pos % self.block_size
            kk = kflat[sl].transpose(0, 1)[None]
            vv = vflat[sl].transpose(0, 1)[None]
            qq = q[a:b].transpose(0, 1)[None]
            if not q.is_cuda:
                qq, kk, vv = qq.float(), kk.float(), vv.float()
            mask = (torch.arange(total, device=q.device)[None, :] <=
                    (torch.arange(n_new, device=q.device)[:, None] + start))
            o = F.scaled_dot_product_attention(qq, kk.to(qq.dtype), vv.to(qq.dtype), attn_mask=mask,
                                               scale=self.scale, enable_gqa=(cfg.n_heads != cfg.n_kv_heads))
            attn[a:b] = o[0].transpose(0, 1).to(attn.dtype)

    def _row_parallel(self, a, W, x):
        """x += a @ W^T, summed over TP ranks (prefill): the ordered two-shot all-reduce over
        NVLink peer memory (each chunk's f32 partial written straight into the symmetric
        region by the GEMM), or NCCL for the baseline."""
        if self.tp is None:
            ops.linear(a, W, x, ops.GEMV_ADD_F32)
            return
        if self.tp.fused:
            self.tp.allreduce_rows(a.shape[0], lambda r0, r1, out: ops.linear(a[r0:r1], W, out, ops.GEMV_STORE), x)
            return
        import torch.distributed as dist
        part = torch.zeros_like(x)
        ops.linear(a, W, part, ops.GEMV_ADD_F32)
        dist.all_reduce(part, group=self.tp.ctx.group)
        x.add_(part)

    def _moe_prefill(self, L, h, x):
        """MoE FFN for a prefill chunk: routing on the device, then the local experts over
        their gathered rows (one weight read per active expert), combined in ascending
        expert order; under expert parallelism the NCCL all-gather/reduce-scatter path; under
        tensor parallelism (experts split along their width) the partial outputs are summed
        over the group by the two-shot all-reduce (NCCL for the baseline)."""
        if self.tp is not None and self.tp.fused:
            def partial(r0, r1, out):
                out.zero_()
                self._moe_prefill_local(L, h[r0:r1], out)
            self.tp.allreduce_rows(h.shape[0], partial, x)
            return
        if self.tp is not None:
            import torch.distributed as dist
            part = torch.zeros_like(x)
            self._moe_prefill_local(L, h, part)
            dist.all_reduce(part, group=self.tp.ctx.group)
            x.add_(part)
            return
        self._moe_prefill_local(L, h, x)

    def _moe_prefill_local(self, L, h, x):
        cfg = self.cfg
        T = h.shape[0]
        E, k = cfg.n_experts, cfg.top_k
        dev = h.device
        mb = {"topk_ids": torch.empty(T, k, dtype=torch.int32, device=dev),
              "topk_w": torch.empty(T, k, dtype=torch.float32, device=dev),
              "tok_off": torch.empty(E + 1, dtype=torch.int32, device=dev),
              "tok_idx": torch.empty(T * k, dtype=torch.int32, device=dev),
              "pair_w": torch.empty(T * k, dtype=torch.float32, device=dev),
              "pair_of": torch.empty(T, k, dtype=torch.int32, device=dev), "pred_mask": None}
        if T == 0:
            pass
        elif self.is_cuda:
            if T <= 256:
                logits = torch.empty(T, E, dtype=torch.float32, device=dev)
                ops.router_logits(h, L.router, logits)
            else:  # a plain bf16 GEMM with f32 output (library); top-k and CSR are ours
                logits = torch.mm(h, L.router.t(), out_dtype=torch.float32)
            ops.moe_topk(logits, cfg, L.router_bias, False, mb, counts=self._counts_for(L))
            self._stamp("prefill_moe_route")
        else:
            logits = h.float() @ L.router.float().t()
            _route_torch(logits, cfg, L.router_bias, mb)
            c = self._counts_for(L)
            if c is not None:
                c += torch.bincount(mb["topk_ids"].reshape(-1).long(), minlength=E).to(c.dtype)
        gu, dn = L.experts_gu, L.experts_down
        if L.shared_gu is not None and T > 0:
            x.add_(self._shared_expert(L, h))
        staged = self.expert_cache.staged_ptrs(L) if self.expert_cache is not None else None
        self._stamp("prefill_moe_stage")  # (profiled passes) the wait for this layer's staged host experts
        if self.ep is not None:
            x.add_(self.ep.moe_baseline(h, mb["topk_ids"], mb["topk_w"], gu, dn, staged=staged))
            return
        bk = getattr(gu, "bank_contiguous", False)
        if self.is_cuda and T * k > 256 and gu.qw is not None and gu.e0 == 0 and gu.E == E and \
                gu.N % 128 == 0 and dn.N % 128 == 0 and (bk or staged is not None):
            # every pair is local: rows gathered per expert (CSR from the routing kernel), two
            # grouped tcgen05 GEMMs, then the ordered combine adds the pairs into x
            (gq, gs), (dq, ds) = staged if staged is not None else ((gu.qw_ptrs, gu.sm_ptrs),
                                                                    (dn.qw_ptrs, dn.sm_ptrs))
            P = T * k
            a_rows = h.index_select(0, mb["tok_idx"])
            mid = torch.empty(P, gu.N // 2, dtype=h.dtype, device=dev)
            yp = torch.empty(P, dn.N, dtype=torch.float32, device=dev)
            banks = self.expert_cache.staged_banks(L) if staged is not None and not bk else None
            if banks is not None:
                # residents and staged host experts in two contiguous banks: packed weights by TMA
                gb, db, sel = banks
                ops.core.gemm_grouped_banks(a_rows, mb["tok_off"], gu.N, gu.K, 1, None, mid, gb, sel)
                ops.core.gemm_grouped_banks(mid, mb["tok_off"], dn.N, dn.K, 2, mb["pair_w"], yp, db, sel)
            else:
                ops.gemm_grouped(a_rows, gq, gs, mb["tok_off"], gu.N, gu.K, 1, None, mid, E,
                                 gu.qw if bk else None, gu.sm if bk else None)
                ops.gemm_grouped(mid, dq, ds, mb["tok_off"], dn.N, dn.K, 2, mb["pair_w"], yp, E,
                                 dn.qw if bk else None, dn.sm if bk else None)
            self._stamp("prefill_moe_experts")
            ops.moe_combine_rmsnorm(x, yp, mb["pair_of"], None, None, None, cfg.rms_eps)
            return
        from ..parallel.ep import _local_experts_apply
        x.add_(_local_experts_apply(h, mb["topk_ids"], mb["topk_w"], gu, dn, (gu.e0, gu.e0 + gu.E), staged))


_OFF1: dict = {}


def _off1(n, dev):
    key = (n, str(dev))
    t = _OFF1.get(key)
    if t is None:
        t = torch.tensor([0, n], dtype=torch.int32, device=dev)
        _OFF1[key] = t
    return t


def _route_torch(logits, cfg, bias, mb):
    """Large-T routing with torch ops (same rule as the kernel: ties to the lower index)."""
    T = logits.shape[0]
    E, k = cfg.n_experts, cfg.top_k
    dev = logits.device
    if cfg.router_scoring == "softmax":
        scores = torch.softmax(logits.float(), -1)
        sel = scores
    else:
        scores = torch.sigmoid(logits.float())
        sel = scores + (bias if bias is not None else 0)
    if cfg.n_groups > 1:
        gs = sel.view(T, cfg.n_groups, E // cfg.n_groups)
        gscore = gs.topk(2, -1).values.sum(-1) if cfg.router_scoring == "sigmoid" else gs.max(-1).values
        gi = torch.sort(-gscore, dim=-1, stable=True).indices[:, : cfg.topk_groups]
        gm = torch.zeros_like(gscore).scatter_(1, gi, 1.0)
        sel = sel.masked_fill(gm[:, :, None].expand_as(gs).reshape(T, E) == 0, float("-inf"))
    ids = torch.sort(-sel, dim=-1, stable=True).indices[:, :k]
    w = torch.gather(scores, -1, ids)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    w = w * cfg.routed_scaling
    # pairs sorted by (expert, token); per token choices sorted by expert
    ids_sorted, order = torch.sort(ids, dim=-1)
    w_sorted = torch.gather(w, -1, order)
    flat_e = ids_sorted.reshape(-1)
    key = flat_e.long() * T + torch.arange(T, device=dev).repeat_interleave(k)
    perm = torch.argsort(key)
    counts = torch.bincount(flat_e, minlength=E)
    mb["tok_off"][0] = 0
    mb["tok_off"][1:] = torch.cumsum(counts, 0).int()
    mb["tok_idx"].copy_((perm // k).int())
    mb["pair_w"].copy_(w_sorted.reshape(-1)[perm])
    pair_of = torch.empty(T * k, dtype=torch.int32, device=dev)
    pair_of[perm] = torch.arange(T * k, device=dev, dtype=torch.int32)
    mb["pair_of"].copy_(pair_of.view(T, k))
    mb["topk_ids"].copy_(ids.int())
    mb["topk_w"].copy_(w)
