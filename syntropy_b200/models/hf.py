"""Hugging Face checkpoints: `config.json` -> ModelConfig, and the checkpoint's tensor names ->
this package's canonical state dict.

Accepted architectures (the reference's `llama` and `qwen_moe` families, crates/graph/src/
families/{llama.rs,qwen_moe.rs}): LlamaForCausalLM and MistralForCausalLM (no projection bias,
no sliding window), Qwen2ForCausalLM (bias on the Q, K and V projections), Qwen3ForCausalLM
(QK-norm), Qwen3MoeForCausalLM (QK-norm, every layer MoE).  Rotary scaling other than the
plain one, a sliding window in effect, or an O-projection / MLP bias are rejected with a
message instead of being served wrongly.  Experts may be stored per expert (the Hub layout:
`mlp.experts.{e}.{gate,up,down}_proj.weight`) or fused (`mlp.experts.gate_up_proj`, `down_proj`).
"""
from __future__ import annotations

import json
import os
import re

import torch

from .config import ModelConfig

FAMILY = {"LlamaForCausalLM": "llama", "MistralForCausalLM": "llama", "Qwen2ForCausalLM": "llama",
          "Qwen3ForCausalLM": "llama", "Qwen3MoeForCausalLM": "qwen_moe"}


def config_from_hf(d: dict, name: str = "hf", weight_quant: str = "bf16") -> ModelConfig:
    arch = (d.get("architectures") or ["?"])[0]
    if arch not in FAMILY:
        raise ValueError(f"architecture {arch} is not supported (supported: {sorted(FAMILY)})")
    rope = d.get("rope_scaling") or d.get("rope_parameters") or {}
    rtype = rope.get("rope_type", rope.get("type", "default")) if isinstance(rope, dict) else "default"
    if rtype not in (None, "default"):
        raise ValueError(f"rotary scaling {rtype!r} is not supported")
    theta = d.get("rope_theta") or (rope.get("rope_theta") if isinstance(rope, dict) else None) or 10000.0
    if d.get("use_sliding_window") or (arch == "MistralForCausalLM" and d.get("sliding_window")):
        raise ValueError("sliding-window attention is not supported")
    if d.get("mlp_bias") or (arch != "Qwen2ForCausalLM" and d.get("attention_bias")):
        raise ValueError("O-projection / MLP biases are not supported")
    H, nh = d["hidden_size"], d["num_attention_heads"]
    kw = dict(name=name, family=FAMILY[arch], n_layers=d["num_hidden_layers"], hidden=H, n_heads=nh,
              n_kv_heads=d.get("num_key_value_heads") or nh, head_dim=d.get("head_dim") or H // nh,
              ffn=d.get("intermediate_size") or 0, vocab=d["vocab_size"], rms_eps=d.get("rms_norm_eps", 1e-6),
              rope_theta=float(theta), qk_norm=arch.startswith("Qwen3"), qkv_bias=arch == "Qwen2ForCausalLM",
              tie_embeddings=bool(d.get("tie_word_embeddings", False)), weight_quant=weight_quant)
    if arch == "Qwen3MoeForCausalLM":
        if d.get("mlp_only_layers") or d.get("decoder_sparse_step", 1) != 1:
            raise ValueError("dense layers between the MoE layers are not supported")
        n_exp = d.get("num_experts") or d.get("num_local_experts")  # the key differs between library versions
        kw.update(n_experts=n_exp, top_k=d["num_experts_per_tok"], moe_ffn=d["moe_intermediate_size"],
                  norm_topk_prob=bool(d.get("norm_topk_prob", True)))
    return ModelConfig(**kw)


_LAYER = {"input_layernorm.weight": "attn_norm", "post_attention_layernorm.weight": "ffn_norm",
          "self_attn.q_proj.weight": "q_proj", "self_attn.k_proj.weight": "k_proj",
          "self_attn.v_proj.weight": "v_proj", "self_attn.o_proj.weight": "o_proj",
          "self_attn.q_proj.bias": "q_bias", "self_attn.k_proj.bias": "k_bias", "self_attn.v_proj.bias": "v_bias",
          "self_attn.q_norm.weight": "q_norm", "self_attn.k_norm.weight": "k_norm",
          "mlp.gate_proj.weight": "gate", "mlp.up_proj.weight": "up", "mlp.down_proj.weight": "down",
          "mlp.gate.weight": "router"}


def canonical_from_hf(sd: dict) -> dict:
    """Hugging Face tensor names -> canonical names (experts stacked [E, ...])."""
    out, experts = {}, {}
    for n, t in sd.items():
        if n == "model.embed_tokens.weight":
            out["embed"] = t
        elif n == "model.norm.weight":
            out["final_norm"] = t
        elif n == "lm_head.weight":
            out["lm_head"] = t
        else:
            m = re.fullmatch(r"model\.layers\.(\d+)\.(.+)", n)
            if not m:
                raise KeyError(f"unmapped tensor {n}")
            i, rest = m.groups()
            pre = f"layers.{i}."
            if rest in _LAYER:
                out[pre + _LAYER[rest]] = t
                continue
            e = re.fullmatch(r"mlp\.experts\.(\d+)\.(gate|up|down)_proj\.weight", rest)
            if e:
                experts.setdefault((i, e.group(2)), {})[int(e.group(1))] = t
            elif rest == "mlp.experts.gate_up_proj":  # fused [E, 2f, h]: gate rows, then up rows
                f = t.shape[1] // 2
                out[pre + "experts.gate"], out[pre + "experts.up"] = t[:, :f].contiguous(), t[:, f:].contiguous()
            elif rest == "mlp.experts.down_proj":     # fused [E, h, f]
                out[pre + "experts.down"] = t
            else:
                raise KeyError(f"unmapped tensor {n}")
    for (i, kind), d in experts.items():
        out[f"layers.{i}.experts.{kind}"] = torch.stack([d[e] for e in sorted(d)])
    return out


def load_hf(path: str, weight_quant: str = "bf16", name: str | None = None) -> tuple[ModelConfig, dict]:
    """(config, canonical state dict) of a Hugging Face checkpoint directory."""
    from ..formats.safetensors import load_state_dict
    with open(os.path.join(path, "config.json")) as f:
        cfg = config_from_hf(json.load(f), name or os.path.basename(os.path.normpath(path)), weight_quant)
    return cfg, canonical_from_hf(load_state_dict(path))
