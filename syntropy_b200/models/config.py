"""Model architecture configs.

Families follow the reference's registry (crates/graph/src/families.rs:44): ``llama``
(Llama/Mistral/Qwen2/Qwen3 dense), ``qwen_moe`` (Qwen3-MoE) and ``deepseek3`` (MLA + MoE +
MTP, designed in plan/rfcs/RFC-0043-model-graph-ir-and-architecture-families.md).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field


@dataclass
class ModelConfig:
    name: str
    family: str  # "llama" | "qwen_moe" | "deepseek3"
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int  # dense FFN width
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    # ("llama3", factor, low_freq_factor, high_freq_factor, original_max_positions),
    # ("yarn", factor, original_max_positions, beta_fast, beta_slow, mscale, mscale_all_dim) or () (plain)
    rope_scaling: tuple = ()
    qk_norm: bool = False
    qkv_bias: bool = False  # bias on the Q, K and V projections (Qwen2)
    tie_embeddings: bool = False
    # MoE
    n_experts: int = 0
    top_k: int = 0
    moe_ffn: int = 0
    n_shared_experts: int = 0
    norm_topk_prob: bool = True
    router_scoring: str = "softmax"  # "softmax" | "sigmoid"
    n_groups: int = 1  # group-limited routing (deepseek3)
    topk_groups: int = 1
    routed_scaling: float = 1.0
    first_dense_layers: int = 0  # leading dense layers (deepseek3)
    # MLA (deepseek3)
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_rope_dim: int = 0
    qk_nope_dim: int = 0
    v_head_dim: int = 0
    n_mtp: int = 0
    # storage
    weight_quant: str = "bf16"  # "bf16" | "fp32" | "q4" | "fp8"
    init_std: float = 0.02

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def layer_is_moe(self, i: int) -> bool:
        return self.is_moe and i >= self.first_dense_layers

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def param_count(self) -> int:
        """Parameter count (embeddings and head included)."""
        h = self.hidden
        n = self.vocab * h * (1 if self.tie_embeddings else 2)
        for i in range(self.n_layers):
            if self.is_mla:
                qd = self.n_heads * (self.qk_nope_dim + self.qk_rope_dim)
                attn = (h * self.q_lora_rank + self.q_lora_rank * qd if self.q_lora_rank else h * qd)
                attn += h * (self.kv_lora_rank + self.qk_rope_dim)
                attn += self.kv_lora_rank * self.n_heads * (self.qk_nope_dim + self.v_head_dim)
                attn += self.n_heads * self.v_head_dim * h
            else:
                attn = h * (self.q_dim + 2 * self.kv_dim) + self.q_dim * h
                attn += (self.q_dim + 2 * self.kv_dim) if self.qkv_bias else 0
            if self.layer_is_moe(i):
                ffn = self.n_experts * 3 * h * self.moe_ffn + h * self.n_experts
                ffn += self.n_shared_experts * 3 * h * self.moe_ffn
            else:
                ffn = 3 * h * self.ffn
            n += attn + ffn
        return n

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        """KV bytes stored per token over all layers (reference formula:
        crates/manifest/src/kv.rs:32-188)."""
        if self.is_mla:
            per_layer = (self.kv_lora_rank + self.qk_rope_dim) * dtype_bytes
        else:
            per_layer = 2 * self.kv_dim * dtype_bytes
        return per_layer * self.n_layers


PRESETS: dict[str, ModelConfig] = {}


def _reg(c: ModelConfig) -> ModelConfig:
    PRESETS[c.name] = c
    return c


# Plumbing config (CPU kernels, no GPU).
_reg(ModelConfig(name="tiny-llama", family="llama", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2,
                 head_dim=64, ffn=688, vocab=1024, rms_eps=1e-5, rope_theta=10000.0, weight_quant="fp32"))
_reg(ModelConfig(name="llama3-8b", family="llama", n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8,
                 head_dim=128, ffn=14336, vocab=128256, rms_eps=1e-5, rope_theta=500000.0, weight_quant="bf16"))
_reg(ModelConfig(name="llama3-70b", family="llama", n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8,
                 head_dim=128, ffn=28672, vocab=128256, rms_eps=1e-5, rope_theta=500000.0, weight_quant="q4"))
_reg(ModelConfig(name="qwen3-235b-a22b", family="qwen_moe", n_layers=94, hidden=4096, n_heads=64,
                 n_kv_heads=4, head_dim=128, ffn=12288, vocab=151936, rms_eps=1e-6, rope_theta=1000000.0,
                 qk_norm=True, n_experts=128, top_k=8, moe_ffn=1536, norm_topk_prob=True, weight_quant="q4"))
_reg(ModelConfig(name="deepseek-v3", family="deepseek3", n_layers=61, hidden=7168, n_heads=128,
                 n_kv_heads=128, head_dim=192, ffn=18432, vocab=129280, rms_eps=1e-6, rope_theta=10000.0,
                 n_experts=256, top_k=8, moe_ffn=2048, n_shared_experts=1, norm_topk_prob=True,
                 router_scoring="sigmoid", n_groups=8, topk_groups=4, routed_scaling=2.5, first_dense_layers=3,
                 q_lora_rank=1536, kv_lora_rank=512, qk_rope_dim=64, qk_nope_dim=128, v_head_dim=128, n_mtp=1,
                 weight_quant="fp8"))
# Small same-family configs for tests (same code paths, fewer/smaller layers).
_reg(ModelConfig(name="tiny-qwen2", family="llama", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2,
                 head_dim=64, ffn=512, vocab=1024, rms_eps=1e-6, rope_theta=1000000.0, qkv_bias=True,
                 tie_embeddings=True, weight_quant="fp32"))
_reg(ModelConfig(name="qwen2.5-7b", family="llama", n_layers=28, hidden=3584, n_heads=28, n_kv_heads=4,
                 head_dim=128, ffn=18944, vocab=152064, rms_eps=1e-6, rope_theta=1000000.0, qkv_bias=True,
                 weight_quant="bf16"))
_reg(ModelConfig(name="tiny-qwen-moe", family="qwen_moe", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2,
                 head_dim=64, ffn=512, vocab=1024, rms_eps=1e-6, rope_theta=1000000.0, qk_norm=True,
                 n_experts=8, top_k=2, moe_ffn=128, weight_quant="fp32"))
_reg(ModelConfig(name="small-qwen-moe", family="qwen_moe", n_layers=4, hidden=1024, n_heads=16, n_kv_heads=4,
                 head_dim=128, ffn=2048, vocab=4096, rms_eps=1e-6, rope_theta=1000000.0, qk_norm=True,
                 n_experts=16, top_k=4, moe_ffn=256, weight_quant="q4"))
_reg(ModelConfig(name="small-llama", family="llama", n_layers=4, hidden=1024, n_heads=8, n_kv_heads=2,
                 head_dim=128, ffn=2048, vocab=4096, rms_eps=1e-5, rope_theta=500000.0, weight_quant="q4"))
_reg(ModelConfig(name="small-deepseek", family="deepseek3", n_layers=3, hidden=1024, n_heads=16, n_kv_heads=16,
                 head_dim=192, ffn=2048, vocab=4096, rms_eps=1e-6, rope_theta=10000.0, n_experts=16, top_k=4,
                 moe_ffn=256, n_shared_experts=1, router_scoring="sigmoid", n_groups=4, topk_groups=2,
                 routed_scaling=2.5, first_dense_layers=1, q_lora_rank=256, kv_lora_rank=512, qk_rope_dim=64,
                 qk_nope_dim=128, v_head_dim=128, n_mtp=1, weight_quant="fp8"))
_reg(ModelConfig(name="tiny-deepseek", family="deepseek3", n_layers=3, hidden=256, n_heads=4, n_kv_heads=4,
                 head_dim=96, ffn=512, vocab=1024, rms_eps=1e-6, rope_theta=10000.0, n_experts=8, top_k=2,
                 moe_ffn=128, n_shared_experts=1, router_scoring="sigmoid", n_groups=4, topk_groups=2,
                 routed_scaling=2.5, first_dense_layers=1, q_lora_rank=128, kv_lora_rank=64, qk_rope_dim=32,
                 qk_nope_dim=64, v_head_dim=64, n_mtp=1, weight_quant="fp32"))


def get_config(name: str, **overrides) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model config {name!r}; known: {sorted(PRESETS)}")
    c = PRESETS[name]
    return c.replace(**overrides) if overrides else c
