"""Engine forward for the ``llama`` and ``qwen_moe`` families (GQA attention, dense SwiGLU
or top-k MoE FFN), over paged KV.

Per-layer decode sequence (each line one kernel on CUDA):
    qkv   = gemv(h, Wqkv)                         q4 GEMV
    q     = qk_norm + rope(qkv); k, v -> pages    fused RmsNorm+Rope+KvWrite
    o     = paged_attention(q, pages)             split-KV decode attention + merge
    x    += gemv(o, Wo)                           q4 GEMV, f32 residual epilogue
    h     = rmsnorm(x)
  dense:  a = swiglu(gemv(h, Wgu)); x += gemv(a, Wd)
  MoE:    logits = router(h [, next router]); top-k + CSR
          a  = swiglu(grouped_gemv(h, Wgu[e]))   one weight read per active expert
          yp = w * grouped_gemv(a, Wd[e])
          x += sum_j yp (ascending expert);  h = rmsnorm_next(x)   fused combine
Block structure follows crates/graph/src/blocks/snapshots/{gqa_fused,dense_ffn,moe}.txt.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .. import ops
from ..formats.q4 import Q4Weight
from .config import ModelConfig
from .reference import rope_table
from .weights import expert_tensor, make_tensor, layer_shapes


@dataclass
class ExpertBank:
    """Stacked per-expert matrices [E][N, K].  On CUDA: q4 tiled storage + pointer tables
    (the pointer of expert e may point into the VRAM bank, a cache slot or host memory)."""

    E: int        # experts held (local rows)
    N: int
    K: int
    e0: int = 0   # global id of local row 0 (expert parallelism)
    qw: torch.Tensor | None = None    # int32 [E, N*K/8]
    sm: torch.Tensor | None = None    # fp16 [E, N*K/16]
    w: torch.Tensor | None = None     # CPU/dense: [E, N, K]
    qw_ptrs: torch.Tensor | None = None  # int64 [E] device
    sm_ptrs: torch.Tensor | None = None
    bank_contiguous: bool = False  # qw/sm hold every expert in order (TMA-streamable bank)
    f8: torch.Tensor | None = None   # fp8 experts: uint8 [E, N*K] in the tiled e4m3 layout
    f8s: torch.Tensor | None = None  # f32 [E, ceil(N/128), K/128] block scales

    @property
    def is_fp8(self) -> bool:
        return self.f8 is not None

    def weight(self, e: int) -> torch.Tensor:
        if self.w is not None:
            return self.w[e]
        if self.f8 is not None:
            from ..formats.fp8 import FP8Weight
            return FP8Weight(self.N, self.K, None, self.f8s[e], self.f8[e]).dequant()
        return Q4Weight(self.N, self.K, self.qw[e], self.sm[e]).dequant()

    def build_ptrs(self):
        if self.f8 is not None:
            dev = self.f8.device
            qb, sb = self.f8.data_ptr(), self.f8s.data_ptr()
            qs, ss = self.f8.stride(0), self.f8s.stride(0) * 4
            self.qw_ptrs = torch.tensor([qb + e * qs for e in range(self.E)], dtype=torch.int64, device=dev)
            self.sm_ptrs = torch.tensor([sb + e * ss for e in range(self.E)], dtype=torch.int64, device=dev)
            return
        if self.qw is None:
            return
        self.bank_contiguous = True
        dev = self.qw.device
        qb, sb = self.qw.data_ptr(), self.sm.data_ptr()
        qs, ss = self.qw.stride(0) * 4, self.sm.stride(0) * 2
        self.qw_ptrs = torch.tensor([qb + e * qs for e in range(self.E)], dtype=torch.int64, device=dev)
        self.sm_ptrs = torch.tensor([sb + e * ss for e in range(self.E)], dtype=torch.int64, device=dev)

    @property
    def expert_nbytes(self) -> int:
        if self.f8 is not None:
            return self.N * self.K + self.f8s[0].numel() * 4
        return self.N * self.K // 32 * 20


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    qkv: object
    o: object
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    qkv_bias: torch.Tensor | None = None  # [q_dim + 2 kv_dim] in the activation dtype (Qwen2)
    gate_up: object = None
    down: object = None
    router: torch.Tensor | None = None      # [E, H] (bf16 on CUDA)
    router_cat: torch.Tensor | None = None  # [2E, H]: this layer's rows then the next layer's
    router_bias: torch.Tensor | None = None
    experts_gu: ExpertBank | None = None
    experts_down: ExpertBank | None = None
    is_moe: bool = False
    mla: dict | None = None
    shared_gu: object = None
    shared_down: object = None


@dataclass
class ModelWeights:
    cfg: ModelConfig
    device: torch.device
    embed: torch.Tensor
    final_norm: torch.Tensor
    lm_head: object
    layers: list = field(default_factory=list)
    rope_cos: torch.Tensor | None = None
    rope_sin: torch.Tensor | None = None
    mtp: object = None
    layer_offset: int = 0

    def nbytes(self) -> int:
        tot = 0
        seen = set()

        def add(t):
            nonlocal tot
            if t is None:
                return
            if isinstance(t, Q4Weight) or type(t).__name__ == "FP8Weight":
                tot += t.nbytes
            elif isinstance(t, ExpertBank):
                for x in (t.qw, t.sm, t.w, t.f8, t.f8s):
                    if x is not None and x.data_ptr() not in seen:
                        seen.add(x.data_ptr())
                        tot += x.numel() * x.element_size()
            elif isinstance(t, torch.Tensor):
                tot += t.numel() * t.element_size()

        add(self.embed)
        add(self.lm_head)
        for L in self.layers:
            for v in L.__dict__.values():
                add(v)
        return tot


class _RemapState(dict):
    """Serves "layers.0.<x>" from "<prefix><x>" of an underlying (possibly lazy) state."""

    def __init__(self, base, prefix):
        super().__init__()
        self.base, self.prefix = base, prefix

    def __getitem__(self, name):
        return self.base[name.replace("layers.0.", self.prefix)] if name.startswith("layers.0.") else self.base[name]

    def __contains__(self, name):
        return name.replace("layers.0.", self.prefix) in self.base


def _prepare_mtp(cfg, get, quant, device, base_state, seed, expert_range):
    """The multi-token-prediction head: h' = proj([enorm(emb(t+1)); hnorm(x_t)]) followed by
    one transformer block shaped like the last layer (weights under "mtp.")."""
    h = cfg.hidden
    m = {"enorm": get("mtp.enorm", (h,)).float(), "hnorm": get("mtp.hnorm", (h,)).float(),
         "proj": _linear_weight(get("mtp.proj", (h, 2 * h)), "bf16" if device.type == "cuda" else quant, device)}
    last_moe = cfg.layer_is_moe(cfg.n_layers - 1)
    c1 = cfg.replace(n_layers=1, first_dense_layers=0 if last_moe else 1, n_mtp=0)
    st = _RemapState(base_state, "mtp.block.")
    m["block"] = prepare_weights(c1, device, seed, quant, st, 8, expert_range).layers[0]
    return m


class _LazyState(dict):
    """Canonical state dict whose tensors are generated on first access."""

    def __init__(self, cfg, seed, device):
        super().__init__()
        self.cfg, self.seed, self.device = cfg, seed, device
        from .weights import iter_names
        self.shapes = dict(iter_names(cfg))

    def __getitem__(self, name):
        return make_tensor(self.cfg, name, self.shapes[name], seed=self.seed, device=self.device)

    def __contains__(self, name):
        return name in self.shapes

    def items(self):
        return ((n, self[n]) for n in self.shapes)


class _LazyShard(dict):
    """TP shard of a lazily generated state dict."""

    def __init__(self, full, cfg, rank, size):
        super().__init__()
        self.full, self.cfg, self.rank, self.size = full, cfg, rank, size

    def __getitem__(self, name):
        from ..parallel.tp import shard_state
        return shard_state(self.cfg, {name: self.full[name]}, self.rank, self.size)[name]

    def __contains__(self, name):
        return name in self.full


def _linear_weight(w: torch.Tensor, quant: str, device):
    if device.type == "cuda":
        if quant == "q4":
            return Q4Weight.quantize(w.to(device))
        if quant == "fp8" and w.shape[0] % 16 == 0 and w.shape[1] % 128 == 0:
            from ..formats.fp8 import FP8Weight
            return FP8Weight.quantize(w.to(device))
        return w.to(device=device, dtype=torch.bfloat16)
    return w.float()


def prepare_weights(cfg: ModelConfig, device="cpu", seed: int = 0, quant: str | None = None,
                    state_dict: dict | None = None, max_pos: int = 8192,
                    expert_range: tuple[int, int] | None = None, dense_dtype=None,
                    tp: tuple[int, int] | None = None, layer_range: tuple[int, int] | None = None) -> ModelWeights:
    """Builds engine-ready weights from ``state_dict`` (canonical names) or synthetic ones
    generated directly on ``device``.  ``expert_range`` limits MoE experts to [a, b)
    (expert parallelism).  ``tp=(rank, size)`` keeps this rank's tensor-parallel shard
    (whole heads / FFN columns) and returns weights whose cfg has the local head counts."""
    device = torch.device(device)
    if tp is not None and tp[1] > 1:
        from ..parallel.tp import local_config, shard_state
        from .weights import synthetic_state_dict
        full = state_dict if state_dict is not None else None
        if full is None:
            # generate each tensor on the device, then keep this rank's slice
            full = _LazyState(cfg, seed, device if device.type == "cuda" else "cpu")
        lazy = isinstance(full, _LazyState) or getattr(full, "lazy", False)
        sd_local = _LazyShard(full, cfg, tp[0], tp[1]) if lazy else shard_state(cfg, full, tp[0], tp[1])
        mw = prepare_weights(local_config(cfg, tp[1]), device, seed, quant, sd_local, max_pos, expert_range,
                             dense_dtype, None, layer_range)
        return mw
    quant = quant or cfg.weight_quant
    is_cuda = device.type == "cuda"
    gen_dev = device if is_cuda else "cpu"

    def get(name, shape):
        if state_dict is not None:
            return state_dict[name].to(gen_dev).float()
        return make_tensor(cfg, name, shape, seed=seed, device=gen_dev)

    ea, eb = expert_range if expert_range else (0, cfg.n_experts)
    shapes_g = {"embed": (cfg.vocab, cfg.hidden), "final_norm": (cfg.hidden,), "lm_head": (cfg.vocab, cfg.hidden)}
    emb = get("embed", shapes_g["embed"])
    mw = ModelWeights(
        cfg=cfg, device=device,
        embed=emb.to(torch.bfloat16) if is_cuda else emb,
        final_norm=get("final_norm", shapes_g["final_norm"]).float(),
        lm_head=_linear_weight(emb if cfg.tie_embeddings else get("lm_head", shapes_g["lm_head"]), quant, device),
    )
    del emb
    la, lb = layer_range if layer_range is not None else (0, cfg.n_layers)
    mw.layer_offset = la
    for i in range(la, lb):
        pre = f"layers.{i}."
        sh = layer_shapes(cfg, i)
        if cfg.is_mla:
            from .mla import prepare_mla
            L = LayerWeights(attn_norm=get(pre + "attn_norm", sh["attn_norm"]).float(),
                             ffn_norm=get(pre + "ffn_norm", sh["ffn_norm"]).float(), qkv=None,
                             o=_linear_weight(get(pre + "o_proj", sh["o_proj"]), quant, device))
            L.mla = prepare_mla(cfg, lambda n: get(n, sh[n.split(".")[-1]]), pre,
                                lambda w: _linear_weight(w, quant, device))
        else:
            qkv = torch.cat([get(pre + "q_proj", sh["q_proj"]), get(pre + "k_proj", sh["k_proj"]),
                             get(pre + "v_proj", sh["v_proj"])], 0)
            L = LayerWeights(
                attn_norm=get(pre + "attn_norm", sh["attn_norm"]).float(),
                ffn_norm=get(pre + "ffn_norm", sh["ffn_norm"]).float(),
                qkv=_linear_weight(qkv, quant, device),
                o=_linear_weight(get(pre + "o_proj", sh["o_proj"]), quant, device),
            )
            del qkv
        if cfg.qk_norm:
            L.q_norm = get(pre + "q_norm", sh["q_norm"]).float()
            L.k_norm = get(pre + "k_norm", sh["k_norm"]).float()
        if cfg.qkv_bias and not cfg.is_mla:
            b = torch.cat([get(pre + "q_bias", sh["q_bias"]), get(pre + "k_bias", sh["k_bias"]),
                           get(pre + "v_bias", sh["v_bias"])]).float()
            L.qkv_bias = b.to(device, torch.bfloat16 if is_cuda else torch.float32)
        if cfg.layer_is_moe(i):
            L.is_moe = True
            r = get(pre + "router", sh["router"])
            L.router = r.to(torch.bfloat16) if is_cuda else r
            E, f, H = cfg.n_experts, cfg.moe_ffn, cfg.hidden
            El = eb - ea
            gu = ExpertBank(El, 2 * f, H, e0=ea)
            dn = ExpertBank(El, H, f, e0=ea)
            if is_cuda and quant == "q4":
                gu.qw = torch.zeros(El, 2 * f * H // 8, dtype=torch.int32, device=device)
                gu.sm = torch.zeros(El, 2 * f * H // 16, dtype=torch.float16, device=device)
                dn.qw = torch.zeros(El, H * f // 8, dtype=torch.int32, device=device)
                dn.sm = torch.zeros(El, H * f // 16, dtype=torch.float16, device=device)
                for e in range(ea, eb):
                    if state_dict is not None:
                        g = state_dict[pre + "experts.gate"][e].to(gen_dev).float()
                        u = state_dict[pre + "experts.up"][e].to(gen_dev).float()
                        d = state_dict[pre + "experts.down"][e].to(gen_dev).float()
                    else:
                        g = expert_tensor(cfg, pre + "experts.gate", e, (f, H), seed=seed, device=gen_dev)
                        u = expert_tensor(cfg, pre + "experts.up", e, (f, H), seed=seed, device=gen_dev)
                        d = expert_tensor(cfg, pre + "experts.down", e, (H, f), seed=seed, device=gen_dev)
                    q = Q4Weight.quantize(ops.interleave_gate_up(g, u))
                    gu.qw[e - ea].copy_(q.qw)
                    gu.sm[e - ea].copy_(q.sm)
                    q = Q4Weight.quantize(d)
                    dn.qw[e - ea].copy_(q.qw)
                    dn.sm[e - ea].copy_(q.sm)
                    del g, u, d, q
                gu.build_ptrs()
                dn.build_ptrs()
            elif is_cuda and quant == "fp8" and H % 128 == 0 and f % 128 == 0:
                from ..formats.fp8 import FP8Weight
                gu.f8 = torch.empty(El, 2 * f * H, dtype=torch.uint8, device=device)
                gu.f8s = torch.empty(El, (2 * f + 127) // 128, H // 128, dtype=torch.float32, device=device)
                dn.f8 = torch.empty(El, H * f, dtype=torch.uint8, device=device)
                dn.f8s = torch.empty(El, (H + 127) // 128, f // 128, dtype=torch.float32, device=device)
                for e in range(ea, eb):
                    if state_dict is not None:
                        g = state_dict[pre + "experts.gate"][e].to(gen_dev).float()
                        u = state_dict[pre + "experts.up"][e].to(gen_dev).float()
                        d = state_dict[pre + "experts.down"][e].to(gen_dev).float()
                    else:
                        g = expert_tensor(cfg, pre + "experts.gate", e, (f, H), seed=seed, device=gen_dev)
                        u = expert_tensor(cfg, pre + "experts.up", e, (f, H), seed=seed, device=gen_dev)
                        d = expert_tensor(cfg, pre + "experts.down", e, (H, f), seed=seed, device=gen_dev)
                    q = FP8Weight.quantize(ops.interleave_gate_up(g, u))
                    gu.f8[e - ea].copy_(q.tiled)
                    gu.f8s[e - ea].copy_(q.scale)
                    q = FP8Weight.quantize(d)
                    dn.f8[e - ea].copy_(q.tiled)
                    dn.f8s[e - ea].copy_(q.scale)
                    del g, u, d, q
                gu.build_ptrs()
                dn.build_ptrs()
            elif state_dict is not None:  # expert by expert (a lazy checkpoint reads one at a time)
                G, U, D = (state_dict[pre + "experts." + k] for k in ("gate", "up", "down"))
                gu.w = torch.stack([ops.interleave_gate_up(G[e].to(gen_dev).float(), U[e].to(gen_dev).float())
                                    for e in range(ea, eb)])
                dn.w = torch.stack([D[e].to(gen_dev).float() for e in range(ea, eb)])
                if is_cuda:
                    gu.w = gu.w.to(device=device, dtype=torch.bfloat16)
                    dn.w = dn.w.to(device=device, dtype=torch.bfloat16)
            else:
                g = get(pre + "experts.gate", sh["experts.gate"])
                u = get(pre + "experts.up", sh["experts.up"])
                gu.w = torch.stack([ops.interleave_gate_up(g[e], u[e]) for e in range(ea, eb)])
                dn.w = get(pre + "experts.down", sh["experts.down"])[ea:eb].contiguous()
                if is_cuda:
                    gu.w = gu.w.to(device=device, dtype=torch.bfloat16)
                    dn.w = dn.w.to(device=device, dtype=torch.bfloat16)
            L.experts_gu, L.experts_down = gu, dn
            if "router_bias" in sh:
                L.router_bias = get(pre + "router_bias", sh["router_bias"]).float()
            if cfg.n_shared_experts:
                sgu = ops.interleave_gate_up(get(pre + "shared.gate", sh["shared.gate"]),
                                             get(pre + "shared.up", sh["shared.up"]))
                L.shared_gu = _linear_weight(sgu, quant, device)
                L.shared_down = _linear_weight(get(pre + "shared.down", sh["shared.down"]), quant, device)
        else:
            gu = ops.interleave_gate_up(get(pre + "gate", sh["gate"]), get(pre + "up", sh["up"]))
            L.gate_up = _linear_weight(gu, quant, device)
            L.down = _linear_weight(get(pre + "down", sh["down"]), quant, device)
        mw.layers.append(L)
    # next-layer router rows appended for prediction (the last MoE layer predicts nothing)
    for i, L in enumerate(mw.layers):
        if L.is_moe and i + 1 < len(mw.layers) and mw.layers[i + 1].is_moe:
            L.router_cat = torch.cat([L.router, mw.layers[i + 1].router], 0).contiguous()
    if cfg.n_mtp:
        base = state_dict if state_dict is not None else _LazyState(cfg, seed, gen_dev)
        mw.mtp = _prepare_mtp(cfg, get, quant, device, base, seed, expert_range)
    cos, sin = rope_table(cfg.qk_rope_dim if cfg.is_mla else cfg.head_dim, cfg.rope_theta, max_pos, device,
                          cfg.rope_scaling)
    mw.rope_cos, mw.rope_sin = cos.contiguous(), sin.contiguous()
    return mw
