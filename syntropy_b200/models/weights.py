"""Synthetic weights of a named architecture.

Every tensor is drawn from N(0, init_std) by its own generator, seeded from the model seed
and the tensor name, so any subset (one layer, one rank's experts) can be regenerated
anywhere without materialising the rest.  Norm weights are ones.  Names follow the
canonical scheme below, which the safetensors loader also uses.
"""
from __future__ import annotations

import hashlib
from typing import Iterator

import torch

from .config import ModelConfig


def tensor_seed(seed: int, name: str) -> int:
    h = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") & ((1 << 63) - 1)


def randn(name: str, shape, *, seed: int, std: float, device="cpu", dtype=torch.float32) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(tensor_seed(seed, name))
    t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
    t.mul_(std)
    return t.to(dtype) if dtype != torch.float32 else t


def layer_shapes(cfg: ModelConfig, i: int) -> dict[str, tuple]:
    """Canonical tensor shapes of layer ``i`` (out_features first, like nn.Linear)."""
    h = cfg.hidden
    s: dict[str, tuple] = {"attn_norm": (h,), "ffn_norm": (h,)}
    if cfg.is_mla:
        qd = cfg.n_heads * (cfg.qk_nope_dim + cfg.qk_rope_dim)
        if cfg.q_lora_rank:
            s["q_a"] = (cfg.q_lora_rank, h)
            s["q_a_norm"] = (cfg.q_lora_rank,)
            s["q_b"] = (qd, cfg.q_lora_rank)
        else:
            s["q_proj"] = (qd, h)
        s["kv_a"] = (cfg.kv_lora_rank + cfg.qk_rope_dim, h)
        s["kv_a_norm"] = (cfg.kv_lora_rank,)
        s["kv_b"] = (cfg.n_heads * (cfg.qk_nope_dim + cfg.v_head_dim), cfg.kv_lora_rank)
        s["o_proj"] = (h, cfg.n_heads * cfg.v_head_dim)
    else:
        s["q_proj"] = (cfg.q_dim, h)
        s["k_proj"] = (cfg.kv_dim, h)
        s["v_proj"] = (cfg.kv_dim, h)
        s["o_proj"] = (h, cfg.q_dim)
        if cfg.qkv_bias:
            s["q_bias"] = (cfg.q_dim,)
            s["k_bias"] = (cfg.kv_dim,)
            s["v_bias"] = (cfg.kv_dim,)
        if cfg.qk_norm:
            s["q_norm"] = (cfg.head_dim,)
            s["k_norm"] = (cfg.head_dim,)
    if cfg.layer_is_moe(i):
        E, f = cfg.n_experts, cfg.moe_ffn
        s["router"] = (E, h)
        if cfg.router_scoring == "sigmoid":
            s["router_bias"] = (E,)
        s["experts.gate"] = (E, f, h)
        s["experts.up"] = (E, f, h)
        s["experts.down"] = (E, h, f)
        if cfg.n_shared_experts:
            fs = f * cfg.n_shared_experts
            s["shared.gate"] = (fs, h)
            s["shared.up"] = (fs, h)
            s["shared.down"] = (h, fs)
    else:
        s["gate"] = (cfg.ffn, h)
        s["up"] = (cfg.ffn, h)
        s["down"] = (h, cfg.ffn)
    return s


def is_norm(name: str) -> bool:
    return name.endswith("norm") or name.endswith("_norm")


def expert_tensor(cfg: ModelConfig, full_name: str, e: int, shape, *, seed: int, device="cpu",
                  dtype=torch.float32) -> torch.Tensor:
    """Expert ``e`` of a stacked expert tensor (each expert has its own generator, so an
    expert-parallel rank can build only the experts it owns)."""
    return randn(f"{full_name}.{e}", shape, seed=seed, std=cfg.init_std, device=device, dtype=dtype)


def make_tensor(cfg: ModelConfig, full_name: str, shape, *, seed: int, device="cpu",
                dtype=torch.float32) -> torch.Tensor:
    leaf = full_name.split(".")[-1]
    if is_norm(leaf):
        return torch.ones(shape, device=device, dtype=dtype)
    if leaf == "router_bias":
        return torch.zeros(shape, device=device, dtype=dtype)
    if ".experts." in full_name:
        return torch.stack([expert_tensor(cfg, full_name, e, shape[1:], seed=seed, device=device, dtype=dtype)
                            for e in range(shape[0])])
    return randn(full_name, shape, seed=seed, std=cfg.init_std, device=device, dtype=dtype)


def global_shapes(cfg: ModelConfig) -> dict[str, tuple]:
    s = {"embed": (cfg.vocab, cfg.hidden), "final_norm": (cfg.hidden,)}
    if not cfg.tie_embeddings:
        s["lm_head"] = (cfg.vocab, cfg.hidden)
    if cfg.n_mtp:
        h = cfg.hidden
        s["mtp.enorm"] = (h,)
        s["mtp.hnorm"] = (h,)
        s["mtp.proj"] = (h, 2 * h)
    return s


def iter_names(cfg: ModelConfig) -> Iterator[tuple[str, tuple]]:
    for n, sh in global_shapes(cfg).items():
        yield n, sh
    for i in range(cfg.n_layers):
        for n, sh in layer_shapes(cfg, i).items():
            yield f"layers.{i}.{n}", sh
    if cfg.n_mtp:
        # one extra transformer block for the MTP head (dense-or-MoE like the last layer)
        for n, sh in layer_shapes(cfg, cfg.n_layers - 1).items():
            yield f"mtp.block.{n}", sh


def synthetic_state_dict(cfg: ModelConfig, seed: int = 0, device="cpu", dtype=torch.float32) -> dict:
    """All weights materialised (small configs only)."""
    return {n: make_tensor(cfg, n, sh, seed=seed, device=device, dtype=dtype) for n, sh in iter_names(cfg)}
