"""Naive f32 reference forward: the oracle the engine is checked against.

No KV cache, no paging, no fusion, fixed reduction orders.  Op semantics follow the
reference's F32 reference ops (crates/kernels/src/reference/{norm.rs:63,linear.rs:62-132})
and the MoE combine rule (ascending expert index, f32; plan/rfcs/RFC-0040-kernel-providers-
and-backends.md:419).  Used by the tiny-model tests on CPU and by GPU numerics tests.
"""
from __future__ import annotations

import math

import torch

from .config import ModelConfig


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x32 = x.float()
    return x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps) * w.float()


_ROPE_CACHE: dict = {}


def rope_frequencies(dim: int, theta: float, scaling: tuple = ()) -> torch.Tensor:
    """Inverse frequencies (f64).  ("linear", factor) divides every frequency by `factor`.
    With ("llama3", factor, low, high, original_max_positions),
    the Llama 3.1 rule: wavelengths shorter than original/high keep their frequency, longer
    than original/low are divided by `factor`, and the band between is interpolated linearly
    in original/wavelength between the two."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    if not scaling:
        return inv
    if scaling[0] == "yarn":
        return _yarn_frequencies(dim, theta, *scaling[1:5])
    if scaling[0] == "linear":  # position interpolation: every frequency divided by the factor
        return inv / scaling[1]
    kind, factor, low, high, orig = scaling
    if kind != "llama3":
        raise ValueError(f"rotary scaling {kind!r} is not supported")
    wavelen = 2 * math.pi / inv
    smooth = ((orig / wavelen) - low) / (high - low)
    scaled = torch.where(wavelen > orig / low, inv / factor, inv)
    mid = (wavelen <= orig / low) & (wavelen >= orig / high)
    return torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)


def _yarn_frequencies(dim, theta, factor, orig, beta_fast, beta_slow) -> torch.Tensor:
    """YaRN (Peng et al. 2023): dimensions that rotate more than `beta_fast` times over the
    original context keep their frequency, those that rotate fewer than `beta_slow` times are
    interpolated by `factor`, with a linear ramp over the dimensions in between."""
    base = theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    keep, interp = 1.0 / base, 1.0 / (factor * base)

    def dim_for(rotations):  # the dimension index that completes `rotations` turns in `orig` positions
        return dim * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(theta))
    lo = max(math.floor(dim_for(beta_fast)), 0)
    hi = min(math.ceil(dim_for(beta_slow)), dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = ((torch.arange(dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
    return interp * ramp + keep * (1 - ramp)


def yarn_mscale(factor: float, m: float = 1.0) -> float:
    return 1.0 if factor <= 1 else 0.1 * m * math.log(factor) + 1.0


def rope_magnitude(scaling: tuple = ()) -> float:
    """Factor on cos/sin: YaRN's attention temperature (given, or from mscale / mscale_all_dim),
    else 1."""
    if not scaling or scaling[0] != "yarn":
        return 1.0
    if len(scaling) > 7 and scaling[7]:  # given explicitly
        return scaling[7]
    factor, mscale, mscale_all = scaling[1], scaling[5], scaling[6]
    if mscale and mscale_all:
        return yarn_mscale(factor, mscale) / yarn_mscale(factor, mscale_all)
    return yarn_mscale(factor)


def mla_softmax_scale(cfg: ModelConfig) -> float:
    """1/sqrt(q-k head dim), times mscale(mscale_all_dim)^2 under YaRN (DeepSeek-V3)."""
    s = 1.0 / math.sqrt(cfg.qk_nope_dim + cfg.qk_rope_dim)
    sc = cfg.rope_scaling
    if sc and sc[0] == "yarn" and sc[6]:
        m = yarn_mscale(sc[1], sc[6])
        s *= m * m
    return s


def rope_table(dim: int, theta: float, max_pos: int, device="cpu", scaling: tuple = ()) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_pos, dim/2] in f32, computed in f64 (exact table shared with the kernels)."""
    key = (dim, theta, max_pos, str(device), tuple(scaling))
    t = _ROPE_CACHE.get(key)
    if t is None:
        inv = rope_frequencies(dim, theta, scaling)
        ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
        mag = rope_magnitude(scaling)
        t = ((torch.cos(ang) * mag).float().to(device), (torch.sin(ang) * mag).float().to(device))
        _ROPE_CACHE[key] = t
    return t


def apply_rope(x: torch.Tensor, pos: torch.Tensor, theta: float, scaling: tuple = ()) -> torch.Tensor:
    """Rotate-half RoPE on the last dim. x: [T, H, D], pos: [T]."""
    D = x.shape[-1]
    cos, sin = rope_table(D, theta, int(pos.max().item()) + 1, x.device, scaling)
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    x1, x2 = x[..., : D // 2].float(), x[..., D // 2:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def attention(q, k, v, causal_offset: int = 0):
    """q: [Tq, Hq, D], k/v: [Tk, Hkv, D]; query i sees keys <= i + causal_offset."""
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    g = Hq // Hkv
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) / math.sqrt(D)
    mask = torch.arange(Tk)[None, :] > (torch.arange(Tq)[:, None] + causal_offset)
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, v.float())


def topk_stable(scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k along the last dim; ties go to the lower index (deterministic)."""
    n = scores.shape[-1]
    idx = torch.arange(n, device=scores.device).expand_as(scores)
    # sort by (-score, index): stable sort of -score keeps index order for ties
    order = torch.sort(-scores, dim=-1, stable=True).indices[..., :k]
    del idx
    return torch.gather(scores, -1, order), order


def route(h: torch.Tensor, W: dict, cfg: ModelConfig, pre: str):
    logits = h.float() @ W[pre + "router"].float().t()
    if cfg.router_scoring == "softmax":
        scores = torch.softmax(logits, dim=-1)
        sel_scores = scores
    else:
        scores = torch.sigmoid(logits)
        sel_scores = scores + W[pre + "router_bias"].float()
    if cfg.n_groups > 1:
        T, E = sel_scores.shape
        gs = sel_scores.view(T, cfg.n_groups, E // cfg.n_groups)
        group_score = gs.topk(2, dim=-1).values.sum(-1) if cfg.router_scoring == "sigmoid" else gs.max(-1).values
        _, gidx = topk_stable(group_score, cfg.topk_groups)
        gmask = torch.zeros_like(group_score).scatter_(1, gidx, 1.0)
        smask = gmask[:, :, None].expand_as(gs).reshape(T, E)
        sel_scores = sel_scores.masked_fill(smask == 0, float("-inf"))
    _, ids = topk_stable(sel_scores, cfg.top_k)
    w = torch.gather(scores, -1, ids)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    w = w * cfg.routed_scaling
    return ids, w


def moe(h: torch.Tensor, W: dict, cfg: ModelConfig, pre: str) -> torch.Tensor:
    ids, w = route(h, W, cfg, pre)
    T = h.shape[0]
    out = torch.zeros(T, cfg.hidden, dtype=torch.float32)
    g, u, d = W[pre + "experts.gate"], W[pre + "experts.up"], W[pre + "experts.down"]
    for t in range(T):
        # ascending expert index, f32
        order = torch.argsort(ids[t])
        acc = torch.zeros(cfg.hidden, dtype=torch.float32)
        for j in order.tolist():
            e = int(ids[t, j])
            x = h[t].float()
            a = torch.nn.functional.silu(g[e].float() @ x) * (u[e].float() @ x)
            acc += w[t, j] * (d[e].float() @ a)
        out[t] = acc
    if cfg.n_shared_experts:
        x = h.float()
        a = torch.nn.functional.silu(x @ W[pre + "shared.gate"].float().t()) * (x @ W[pre + "shared.up"].float().t())
        out += a @ W[pre + "shared.down"].float().t()
    return out


def dense_ffn(h, W, pre):
    x = h.float()
    a = torch.nn.functional.silu(x @ W[pre + "gate"].float().t()) * (x @ W[pre + "up"].float().t())
    return a @ W[pre + "down"].float().t()


def gqa_attention_block(h, W, cfg: ModelConfig, pre: str, pos: torch.Tensor, kv_prefix=None):
    T = h.shape[0]
    q = h @ W[pre + "q_proj"].float().t()
    k = h @ W[pre + "k_proj"].float().t()
    v = h @ W[pre + "v_proj"].float().t()
    if cfg.qkv_bias:
        q, k, v = q + W[pre + "q_bias"].float(), k + W[pre + "k_bias"].float(), v + W[pre + "v_bias"].float()
    q = q.view(T, cfg.n_heads, cfg.head_dim)
    k = k.view(T, cfg.n_kv_heads, cfg.head_dim)
    v = v.view(T, cfg.n_kv_heads, cfg.head_dim)
    if cfg.qk_norm:
        q = rms_norm(q, W[pre + "q_norm"], cfg.rms_eps)
        k = rms_norm(k, W[pre + "k_norm"], cfg.rms_eps)
    q = apply_rope(q, pos, cfg.rope_theta, cfg.rope_scaling)
    k = apply_rope(k, pos, cfg.rope_theta, cfg.rope_scaling)
    o = attention(q, k, v)
    return o.reshape(T, -1) @ W[pre + "o_proj"].float().t()


def mla_attention_block(h, W, cfg: ModelConfig, pre: str, pos: torch.Tensor):
    """DeepSeek-V3 multi-head latent attention, naive (non-absorbed) form."""
    T = h.shape[0]
    H, dn, dr, dv = cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
    if cfg.q_lora_rank:
        qa = rms_norm(h @ W[pre + "q_a"].float().t(), W[pre + "q_a_norm"], cfg.rms_eps)
        q = qa @ W[pre + "q_b"].float().t()
    else:
        q = h @ W[pre + "q_proj"].float().t()
    q = q.view(T, H, dn + dr)
    q_nope, q_rope = q[..., :dn], q[..., dn:]
    kva = h @ W[pre + "kv_a"].float().t()
    c, k_rope = kva[:, : cfg.kv_lora_rank], kva[:, cfg.kv_lora_rank:]
    c = rms_norm(c, W[pre + "kv_a_norm"], cfg.rms_eps)
    kv = (c @ W[pre + "kv_b"].float().t()).view(T, H, dn + dv)
    k_nope, v = kv[..., :dn], kv[..., dn:]
    q_rope = apply_rope(q_rope, pos, cfg.rope_theta, cfg.rope_scaling)
    k_rope = apply_rope(k_rope.view(T, 1, dr), pos, cfg.rope_theta, cfg.rope_scaling).expand(T, H, dr)
    qf = torch.cat([q_nope, q_rope], -1)
    kf = torch.cat([k_nope, k_rope], -1)
    s = torch.einsum("qhd,khd->hqk", qf, kf) * mla_softmax_scale(cfg)
    mask = torch.arange(T)[None, :] > torch.arange(T)[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)
    return o.reshape(T, H * dv) @ W[pre + "o_proj"].float().t()


def block(x, W, cfg, pre, pos, i):
    h = rms_norm(x, W[pre + "attn_norm"], cfg.rms_eps)
    if cfg.is_mla:
        x = x + mla_attention_block(h, W, cfg, pre, pos)
    else:
        x = x + gqa_attention_block(h, W, cfg, pre, pos)
    h = rms_norm(x, W[pre + "ffn_norm"], cfg.rms_eps)
    if cfg.layer_is_moe(i):
        x = x + moe(h, W, cfg, pre)
    else:
        x = x + dense_ffn(h, W, pre)
    return x


def forward(tokens: torch.Tensor, W: dict, cfg: ModelConfig, return_hidden: bool = False):
    """tokens: [T] int64 (one sequence from position 0) -> logits [T, vocab] f32."""
    T = tokens.shape[0]
    pos = torch.arange(T)
    x = W["embed"].float()[tokens]
    for i in range(cfg.n_layers):
        x = block(x, W, cfg, f"layers.{i}.", pos, i)
    hidden = x
    y = rms_norm(x, W["final_norm"], cfg.rms_eps)
    head = W["embed"] if cfg.tie_embeddings else W["lm_head"]
    logits = y @ head.float().t()
    return (logits, hidden) if return_hidden else logits


def greedy_generate(prompt: torch.Tensor, W: dict, cfg: ModelConfig, n_new: int) -> list[int]:
    """Greedy decode by re-running the full forward each step (the naive oracle)."""
    toks = prompt.clone()
    out = []
    for _ in range(n_new):
        logits = forward(toks, W, cfg)
        nxt = int(torch.argmax(logits[-1]).item())
        out.append(nxt)
        toks = torch.cat([toks, torch.tensor([nxt])])
    return out
