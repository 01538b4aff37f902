"""Multi-head latent attention (DeepSeek-V3 family) over a paged latent cache, in the
absorbed form: the cache holds per token the normalised KV latent c (kv_lora_rank) and the
rotated shared key k_rope (qk_rope_dim); queries are mapped into latent space with
W_uk, attention runs as one shared "KV head" of width kv_lora+rope, and the latent output
is mapped back per head with W_uv.  Reference: plan/rfcs/RFC-0040-kernel-providers-and-
backends.md `AttnDecode(Mla)` (absorbed form, latent 512 + rope 64); naive f32 oracle in
models/reference.py (mla_attention_block).
"""
from __future__ import annotations


import torch
import torch.nn.functional as F

from .. import ops
from .reference import mla_softmax_scale, rope_table


def prepare_mla(cfg, get, pre, linear_weight):
    """Builds the MLA tensors of one layer from canonical weights."""
    H, dn, dv, C = cfg.n_heads, cfg.qk_nope_dim, cfg.v_head_dim, cfg.kv_lora_rank
    w = {}
    if cfg.q_lora_rank:
        w["q_a"] = linear_weight(get(pre + "q_a"))
        w["q_a_norm"] = get(pre + "q_a_norm").float()
        w["q_b"] = linear_weight(get(pre + "q_b"))
    else:
        w["q_proj"] = linear_weight(get(pre + "q_proj"))
    w["kv_a"] = linear_weight(get(pre + "kv_a"))
    w["kv_a_norm"] = get(pre + "kv_a_norm").float()
    kvb = get(pre + "kv_b").float().view(H, dn + dv, C)
    # [H, dn, C] / [H, dv, C]; bf16 on the GPU (the decode kernels read them once per step, the
    # eager paths widen them to f32 where they use them)
    wt = torch.bfloat16 if kvb.is_cuda else torch.float32
    w["w_uk"] = kvb[:, :dn, :].to(wt).contiguous()
    w["w_uv"] = kvb[:, dn:, :].to(wt).contiguous()
    return w


def mla_qkv_decode(cfg, m, h, pos, slot, cos_t, sin_t, cache, qcat):
    """GPU decode projections for T rows: the latent row (normed c | roped k_pe) goes straight
    into the cache at `slot` (int64; -1 = padding, written to the null page) and qcat (bf16
    [T, H, C + dr]) receives [q_nope . W_uk | roped q_pe] for the latent attention kernel."""
    from .._ext import ext
    T = h.shape[0]
    H, dn, dr, C = cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.kv_lora_rank
    q = torch.empty(T, H * (dn + dr), dtype=torch.bfloat16, device=h.device)
    if cfg.q_lora_rank:
        qa = torch.empty(T, cfg.q_lora_rank, dtype=torch.bfloat16, device=h.device)
        ops.linear(h, m["q_a"], qa, ops.GEMV_STORE)
        qa = ops.rms_norm(qa, m["q_a_norm"], cfg.rms_eps)
        ops.linear(qa.to(torch.bfloat16), m["q_b"], q, ops.GEMV_STORE)
    else:
        ops.linear(h, m["q_proj"], q, ops.GEMV_STORE)
    kva = torch.empty(T, C + dr, dtype=torch.bfloat16, device=h.device)
    ops.linear(h, m["kv_a"], kva, ops.GEMV_STORE)
    e = ext()
    e.mla_kv_write(kva, m["kv_a_norm"], cfg.rms_eps, cos_t, sin_t, pos, slot, cache)
    e.mla_q_absorb(q, m["w_uk"], cos_t, sin_t, pos, qcat)
    ops.core._launched(2)
    return qcat


def _rope(x, pos, theta, cos_t=None, sin_t=None):
    D = x.shape[-1]
    if cos_t is None:
        cos_t, sin_t = rope_table(D, theta, int(pos.max().item()) + 1, x.device)
    c = cos_t[pos.long()][:, None, :]
    s = sin_t[pos.long()][:, None, :]
    a, b = x[..., : D // 2].float(), x[..., D // 2:].float()
    return torch.cat([a * c - b * s, b * c + a * s], -1)


def mla_qkv(cfg, m, h, pos, cos_t, sin_t):
    """Projections for T rows: returns (q_lat [T,H,C], q_pe [T,H,dr], latent row [T, C+dr])."""
    T = h.shape[0]
    H, dn, dr, C = cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.kv_lora_rank
    dt = torch.float32
    if cfg.q_lora_rank:
        qa = torch.empty(T, cfg.q_lora_rank, dtype=h.dtype, device=h.device)
        ops.linear(h, m["q_a"], qa, ops.GEMV_STORE)
        qa = ops.rms_norm(qa.float() if not qa.is_cuda else qa, m["q_a_norm"], cfg.rms_eps)
        q = torch.empty(T, H * (dn + dr), dtype=h.dtype, device=h.device)
        ops.linear(qa.to(h.dtype), m["q_b"], q, ops.GEMV_STORE)
    else:
        q = torch.empty(T, H * (dn + dr), dtype=h.dtype, device=h.device)
        ops.linear(h, m["q_proj"], q, ops.GEMV_STORE)
    q = q.view(T, H, dn + dr).to(dt)
    kva = torch.empty(T, C + dr, dtype=h.dtype, device=h.device)
    ops.linear(h, m["kv_a"], kva, ops.GEMV_STORE)
    kva = kva.to(dt)
    c = kva[:, :C]
    c = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * m["kv_a_norm"]
    k_pe = _rope(kva[:, C:].view(T, 1, dr), pos, cfg.rope_theta, cos_t, sin_t)[:, 0]
    q_pe = _rope(q[..., dn:], pos, cfg.rope_theta, cos_t, sin_t)
    q_lat = torch.einsum("thd,hdc->thc", q[..., :dn], m["w_uk"].to(dt))
    return q_lat, q_pe, torch.cat([c, k_pe], -1)


def mla_attend(cfg, m, q_lat, q_pe, lat, ctx_start: int, causal_from: int | None = None):
    """Attention of queries (rows at positions causal_from.. ) over latent rows lat [S, C+dr]."""
    C = cfg.kv_lora_rank
    scale = mla_softmax_scale(cfg)
    lat = lat.float()
    s = (torch.einsum("thc,sc->ths", q_lat, lat[:, :C]) + torch.einsum("thr,sr->ths", q_pe, lat[:, C:])) * scale
    if causal_from is not None:
        S = lat.shape[0]
        T = q_lat.shape[0]
        mask = torch.arange(S, device=lat.device)[None, :] > (torch.arange(T, device=lat.device)[:, None] + causal_from)
        s = s.masked_fill(mask[:, None, :], float("-inf"))
    p = torch.softmax(s, -1)
    o_lat = torch.einsum("ths,sc->thc", p, lat[:, :C])
    return torch.einsum("thc,hvc->thv", o_lat, m["w_uv"].float()).reshape(q_lat.shape[0], -1)


class MLACache:
    """Paged latent cache: per layer [num_blocks, block_size, C + dr]."""

    def __init__(self, n_layers, num_blocks, width, block_size=16, dtype=torch.bfloat16, device="cpu"):
        self.lat = [torch.zeros(num_blocks, block_size, width, dtype=dtype, device=device) for _ in range(n_layers)]
        self.block_size = block_size

    def write(self, layer, slots: torch.Tensor, rows: torch.Tensor):
        flat = self.lat[layer].view(-1, self.lat[layer].shape[-1])
        ok = slots >= 0
        flat[slots[ok].long()] = rows[ok].to(flat.dtype)

    def gather(self, layer, blocks: torch.Tensor, n: int) -> torch.Tensor:
        bs = self.block_size
        pos = torch.arange(n, device=blocks.device)
        sl = blocks[pos // bs].long() * bs + pos % bs
        return self.lat[layer].view(-1, self.lat[layer].shape[-1])[sl]
