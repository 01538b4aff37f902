"""Hugging Face checkpoints: `config.json` -> ModelConfig, and the checkpoint's tensor names ->
this package's canonical state dict.

Accepted architectures (the reference's `llama` and `qwen_moe` families, crates/graph/src/
families/{llama.rs,qwen_moe.rs}, and the DeepSeek-V3 family of the target configs):
LlamaForCausalLM and MistralForCausalLM (no projection bias, no sliding window),
Qwen2ForCausalLM (bias on the Q, K and V projections), Qwen3ForCausalLM (QK-norm),
Qwen3MoeForCausalLM (QK-norm, every layer MoE), DeepseekV3ForCausalLM (MLA, sigmoid
group-limited routing with a selection bias, shared experts, leading dense layers; its rotary
dimensions, stored interleaved, are reordered to the rotate-half layout used here).  Rotary
scaling other than the plain one, Llama 3.1's "llama3" rule and DeepSeek-V3's YaRN, a sliding
window in effect, or an O-projection / MLP bias are rejected with a message instead of being
served wrongly.
Experts may be stored per expert (the Hub layout: `mlp.experts.{e}.{gate,up,down}_proj.weight`)
or fused (`mlp.experts.gate_up_proj`, `down_proj`).
"""
from __future__ import annotations

import json
import os
import re

import torch

from .config import ModelConfig

FAMILY = {"LlamaForCausalLM": "llama", "MistralForCausalLM": "llama", "Qwen2ForCausalLM": "llama",
          "Qwen3ForCausalLM": "llama", "Qwen3MoeForCausalLM": "qwen_moe", "DeepseekV3ForCausalLM": "deepseek3"}


def config_from_hf(d: dict, name: str = "hf", weight_quant: str = "bf16") -> ModelConfig:
    arch = (d.get("architectures") or ["?"])[0]
    if arch not in FAMILY:
        raise ValueError(f"architecture {arch} is not supported (supported: {sorted(FAMILY)})")
    rope = d.get("rope_scaling") or d.get("rope_parameters") or {}
    rtype = rope.get("rope_type", rope.get("type", "default")) if isinstance(rope, dict) else "default"
    scaling = ()
    if rtype == "yarn":  # DeepSeek-V3 (also scales the MLA softmax) and GQA models (cos/sin only)
        if rope.get("truncate", True) is False:
            raise ValueError("YaRN without truncated correction bounds is not supported")
        if not (rope.get("original_max_position_embeddings") or d.get("max_position_embeddings")):
            raise ValueError("YaRN rotary scaling needs original_max_position_embeddings")
        scaling = ("yarn", float(rope["factor"]),
                   float(rope.get("original_max_position_embeddings") or d.get("max_position_embeddings")),
                   float(rope.get("beta_fast") or 32.0), float(rope.get("beta_slow") or 1.0),
                   float(rope.get("mscale", 1.0) or 0.0), float(rope.get("mscale_all_dim", 0.0) or 0.0),
                   float(rope.get("attention_factor") or 0.0))
    elif rtype == "llama3" and arch != "DeepseekV3ForCausalLM":
        scaling = ("llama3", float(rope["factor"]), float(rope.get("low_freq_factor", 1.0)),
                   float(rope.get("high_freq_factor", 4.0)), float(rope["original_max_position_embeddings"]))
    elif rtype == "linear":
        scaling = ("linear", float(rope["factor"]))
    elif rtype not in (None, "default"):
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
              tie_embeddings=bool(d.get("tie_word_embeddings", False)), weight_quant=weight_quant,
              rope_scaling=scaling)
    if arch == "DeepseekV3ForCausalLM":
        dn, dr, dv = d["qk_nope_head_dim"], d["qk_rope_head_dim"], d["v_head_dim"]
        kw.update(n_kv_heads=nh, head_dim=dn + dr, qk_norm=False, q_lora_rank=d.get("q_lora_rank") or 0,
                  kv_lora_rank=d["kv_lora_rank"], qk_rope_dim=dr, qk_nope_dim=dn, v_head_dim=dv,
                  n_experts=d["n_routed_experts"], top_k=d["num_experts_per_tok"],
                  moe_ffn=d["moe_intermediate_size"], n_shared_experts=d.get("n_shared_experts") or 0,
                  router_scoring="sigmoid", n_groups=d.get("n_group") or 1, topk_groups=d.get("topk_group") or 1,
                  routed_scaling=float(d.get("routed_scaling_factor", 1.0)),
                  norm_topk_prob=bool(d.get("norm_topk_prob", True)),
                  first_dense_layers=d.get("first_k_dense_replace") or 0)
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
          "mlp.gate.weight": "router", "mlp.gate.e_score_correction_bias": "router_bias",
          "mlp.shared_experts.gate_proj.weight": "shared.gate", "mlp.shared_experts.up_proj.weight": "shared.up",
          "mlp.shared_experts.down_proj.weight": "shared.down",
          "self_attn.q_a_proj.weight": "q_a", "self_attn.q_a_layernorm.weight": "q_a_norm",
          "self_attn.q_b_proj.weight": "q_b", "self_attn.kv_a_proj_with_mqa.weight": "kv_a",
          "self_attn.kv_a_layernorm.weight": "kv_a_norm", "self_attn.kv_b_proj.weight": "kv_b"}


def _deinterleave_rope(sd: dict, cfg: ModelConfig):
    """Rotary dimensions stored as interleaved pairs (0,1), (2,3), ... -> rotate-half order
    (evens, then odds) in the rows of the Q projection (per head) and of the shared K rope."""
    dn, dr, H, c = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.n_heads, cfg.kv_lora_rank
    perm = torch.cat([torch.arange(0, dr, 2), torch.arange(1, dr, 2)])
    for n in list(sd):
        leaf = n.split(".")[-1]
        if leaf in ("q_b", "q_proj"):
            w = sd[n].view(H, dn + dr, -1)
            sd[n] = torch.cat([w[:, :dn], w[:, dn:][:, perm]], 1).reshape(H * (dn + dr), -1).contiguous()
        elif leaf == "kv_a":
            w = sd[n]
            sd[n] = torch.cat([w[:c], w[c:][perm]], 0).contiguous()


def canonical_from_hf(sd: dict, cfg: ModelConfig | None = None, rope_interleave: bool = True) -> dict:
    """Hugging Face tensor names -> canonical names (experts stacked [E, ...]; MLA rotary rows
    reordered when `cfg` is an MLA model stored with interleaved rotary dimensions)."""
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
    if cfg is not None and cfg.is_mla and rope_interleave:
        _deinterleave_rope(out, cfg)
    return out


def load_hf(path: str, weight_quant: str = "bf16", name: str | None = None) -> tuple[ModelConfig, dict]:
    """(config, canonical state dict) of a Hugging Face checkpoint directory."""
    from ..formats.safetensors import load_state_dict
    with open(os.path.join(path, "config.json")) as f:
        d = json.load(f)
    cfg = config_from_hf(d, name or os.path.basename(os.path.normpath(path)), weight_quant)
    return cfg, canonical_from_hf(load_state_dict(path), cfg, bool(d.get("rope_interleave", True)))


# ---------------------------------------------------------------------- GGUF checkpoints
_GGUF_ARCH = {"llama": "LlamaForCausalLM", "qwen2": "Qwen2ForCausalLM", "qwen3": "Qwen3ForCausalLM",
              "qwen3moe": "Qwen3MoeForCausalLM"}
_GGUF_LAYER = {"attn_norm": "attn_norm", "ffn_norm": "ffn_norm", "attn_q": "q_proj", "attn_k": "k_proj",
               "attn_v": "v_proj", "attn_output": "o_proj", "attn_q_norm": "q_norm", "attn_k_norm": "k_norm",
               "ffn_gate": "gate", "ffn_up": "up", "ffn_down": "down", "ffn_gate_inp": "router",
               "ffn_gate_exps": "experts.gate", "ffn_up_exps": "experts.up", "ffn_down_exps": "experts.down"}


def _rows_to_rotate_half(w: torch.Tensor, n_heads: int) -> torch.Tensor:
    """llama.cpp stores the Q / K rows of `llama` models with rotary pairs interleaved; per head
    put the even rows first, then the odd ones (the rotate-half order used here)."""
    rows = w.shape[0]
    hd = rows // n_heads
    perm = torch.cat([torch.arange(0, hd, 2), torch.arange(1, hd, 2)])
    return w.reshape(n_heads, hd, *w.shape[1:])[:, perm].reshape(w.shape).contiguous()


def _gguf_config(f, name: str, weight_quant: str) -> tuple[str, ModelConfig]:
    m = f.meta
    arch = m["general.architecture"]
    if arch not in _GGUF_ARCH:
        raise ValueError(f"GGUF architecture {arch!r} is not supported (supported: {sorted(_GGUF_ARCH)})")
    if "rope_freqs.weight" in f.tensors or m.get(f"{arch}.rope.scaling.type", "none") not in ("none", None):
        raise ValueError("rotary scaling in a GGUF file is not supported")
    k = lambda key, default=None: m.get(f"{arch}.{key}", default)  # noqa: E731
    emb_dims = f.tensors["token_embd.weight"][1]
    d = {"architectures": [_GGUF_ARCH[arch]], "hidden_size": int(k("embedding_length")),
         "num_hidden_layers": int(k("block_count")), "num_attention_heads": int(k("attention.head_count")),
         "num_key_value_heads": int(k("attention.head_count_kv", k("attention.head_count"))),
         "intermediate_size": int(k("feed_forward_length", 0) or 0), "vocab_size": int(emb_dims[1]),
         "rms_norm_eps": float(k("attention.layer_norm_rms_epsilon", 1e-6)),
         "rope_theta": float(k("rope.freq_base", 10000.0)),
         "tie_word_embeddings": "output.weight" not in f.tensors}
    if k("attention.key_length"):
        d["head_dim"] = int(k("attention.key_length"))
    if arch == "qwen3moe":
        d.update(num_experts=int(k("expert_count")), num_experts_per_tok=int(k("expert_used_count")),
                 moe_intermediate_size=int(k("expert_feed_forward_length")), norm_topk_prob=True)
    return arch, config_from_hf(d, name, weight_quant)


class GGUFCheckpoint(dict):
    """Canonical-name view of a GGUF file (llama / qwen2 / qwen3 / qwen3moe) whose tensors are
    dequantised when asked for (stacked experts one expert at a time), so weights are prepared
    without the whole f32 model in host memory; `prepare_weights` requantises them as configured.
    llama.cpp's interleaved Q / K rotary rows of `llama` models are put back in rotate-half order."""

    lazy = True

    def __init__(self, path: str, weight_quant: str = "bf16", name: str | None = None):
        super().__init__()
        from ..formats.gguf import GGUFFile
        self.file = f = GGUFFile(path)
        try:
            self.arch, self.cfg = _gguf_config(f, name or os.path.splitext(os.path.basename(path))[0], weight_quant)
            self._map = {}
            for n in f.tensors:
                if n in ("token_embd.weight", "output_norm.weight", "output.weight"):
                    self._map[{"token_embd.weight": "embed", "output_norm.weight": "final_norm",
                               "output.weight": "lm_head"}[n]] = (n, None)
                    continue
                mm = re.fullmatch(r"blk\.(\d+)\.(\w+)\.(weight|bias)", n)
                if not mm or mm.group(2) not in _GGUF_LAYER:
                    raise KeyError(f"unmapped GGUF tensor {n}")
                i, part, kind = mm.groups()
                leaf, rot = _GGUF_LAYER[part], None
                if kind == "bias":
                    leaf = {"q_proj": "q_bias", "k_proj": "k_bias", "v_proj": "v_bias"}[leaf]
                elif self.arch == "llama" and leaf in ("q_proj", "k_proj"):
                    rot = self.cfg.n_heads if leaf == "q_proj" else self.cfg.n_kv_heads
                self._map[f"layers.{i}.{leaf}"] = (n, rot)
        except Exception:
            f.close()
            raise

    def __getitem__(self, name):
        n, rot = self._map[name]
        if name.split(".")[-2:-1] == ["experts"]:
            shape = tuple(reversed(self.file.tensors[n][1]))
            return _ExpertStack(lambda e, n=n: self.file.get_row(n, e), shape[0], shape[1:])
        t = self.file.get(n)
        return _rows_to_rotate_half(t, rot) if rot else t

    def __contains__(self, name):
        return name in self._map

    def __len__(self):
        return len(self._map)

    def __iter__(self):
        return iter(self._map)

    def keys(self):
        return list(self._map)

    def items(self):
        return ((n, self[n]) for n in self._map)

    def close(self):
        self.file.close()


def load_gguf(path: str, weight_quant: str = "bf16", name: str | None = None,
              lazy: bool = False) -> tuple[ModelConfig, dict]:
    """(config, canonical state dict) of a GGUF file: dequantised in full, or with `lazy` the
    `GGUFCheckpoint` view that dequantises tensor by tensor (close it when done)."""
    ck = GGUFCheckpoint(path, weight_quant, name)
    if lazy:
        return ck.cfg, ck
    try:
        return ck.cfg, {n: ck.file.get(ck._map[n][0]) if n.split(".")[-2:-1] == ["experts"] else ck[n]
                        for n in ck.keys()}
    finally:
        ck.close()


# ---------------------------------------------------------------------- lazy loading
class _ExpertStack:
    """Stacked expert tensor [E, ...] read one expert at a time.  A leading-`:` slice (a
    tensor-parallel shard, `t[:, a:b]` or `t[:, :, a:b]`) is kept and applied to each expert."""

    def __init__(self, fetch, n: int, shape: tuple, index: tuple = ()):
        self.fetch, self.n, self._shape, self.index = fetch, n, tuple(shape), index

    @property
    def shape(self):
        return (self.n,) + self._shape

    def __len__(self):
        return self.n

    def __getitem__(self, idx):
        if isinstance(idx, int):
            t = self.fetch(idx)
            return t[self.index] if self.index else t
        if isinstance(idx, tuple) and len(idx) > 1 and idx[0] == slice(None) and not self.index:
            rest = idx[1:]
            shape = list(self._shape)
            for d, s in enumerate(rest):
                shape[d] = len(range(*s.indices(shape[d])))
            return _ExpertStack(self.fetch, self.n, tuple(shape), rest)
        raise TypeError(f"unsupported expert-stack index {idx!r}")


class LazyCheckpoint(dict):
    """Canonical-name view of a Hugging Face safetensors checkpoint whose tensors are read from
    the memory-mapped files when asked for (experts one at a time), so preparing a model larger
    than host memory holds about one tensor at a time.  `lazy` tells `prepare_weights` to shard
    tensor-parallel slices on access instead of slicing the whole dict up front."""

    lazy = True

    def __init__(self, path: str, cfg: ModelConfig, rope_interleave: bool = True):
        super().__init__()
        from ..formats.safetensors import SafetensorsFile
        self.cfg = cfg
        files = sorted(os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
        self._files = [SafetensorsFile(p) for p in files]
        self._where = {n: f for f in self._files for n in f.keys()}
        self._map, self._experts, self._fused = {}, {}, {}
        for n in self._where:
            if n == "model.embed_tokens.weight":
                self._map["embed"] = n
            elif n == "model.norm.weight":
                self._map["final_norm"] = n
            elif n == "lm_head.weight":
                self._map["lm_head"] = n
            else:
                m = re.fullmatch(r"model\.layers\.(\d+)\.(.+)", n)
                if not m:
                    raise KeyError(f"unmapped tensor {n}")
                i, rest = m.groups()
                if rest in _LAYER:
                    self._map[f"layers.{i}.{_LAYER[rest]}"] = n
                    continue
                e = re.fullmatch(r"mlp\.experts\.(\d+)\.(gate|up|down)_proj\.weight", rest)
                if e:
                    self._experts.setdefault(f"layers.{i}.experts.{e.group(2)}", {})[int(e.group(1))] = n
                elif rest == "mlp.experts.gate_up_proj":   # fused [E, 2f, h]: gate rows, then up rows
                    self._fused[f"layers.{i}.experts.gate"] = (n, 0)
                    self._fused[f"layers.{i}.experts.up"] = (n, 1)
                elif rest == "mlp.experts.down_proj":      # fused [E, h, f]
                    self._fused[f"layers.{i}.experts.down"] = (n, None)
                else:
                    raise KeyError(f"unmapped tensor {n}")
        for name, ids in self._experts.items():
            if sorted(ids) != list(range(len(ids))):
                raise KeyError(f"{name}: experts {sorted(set(range(max(ids) + 1)) - set(ids))} missing")
        self._rope = cfg.is_mla and rope_interleave

    def _read(self, hf_name: str) -> torch.Tensor:
        return self._where[hf_name].get(hf_name)

    def _fused_row(self, hf_name: str, half, e: int) -> torch.Tensor:
        t = self._where[hf_name].get_row(hf_name, e)
        if half is None:
            return t
        f = t.shape[0] // 2
        return t[half * f:(half + 1) * f]

    def __getitem__(self, name):
        if name in self._experts:
            ids = self._experts[name]
            shape = tuple(self._where[ids[0]].tensors[ids[0]][1])
            return _ExpertStack(lambda e, ids=ids: self._read(ids[e]), len(ids), shape)
        if name in self._fused:
            n, half = self._fused[name]
            shape = list(self._where[n].tensors[n][1])
            if half is not None:
                shape[1] //= 2
            return _ExpertStack(lambda e, n=n, half=half: self._fused_row(n, half, e), shape[0], tuple(shape[1:]))
        t = self._read(self._map[name])
        if self._rope and name.split(".")[-1] in ("q_b", "q_proj", "kv_a"):
            d = {name: t}
            _deinterleave_rope(d, self.cfg)
            t = d[name]
        return t

    def __contains__(self, name):
        return name in self._map or name in self._experts or name in self._fused

    def __len__(self):
        return len(self._map) + len(self._experts) + len(self._fused)

    def __iter__(self):
        return iter(self.keys())

    def keys(self):
        return list(self._map) + list(self._experts) + list(self._fused)

    def items(self):
        return ((n, self[n]) for n in self.keys())

    def close(self):
        for f in self._files:
            f.close()


def load_hf_lazy(path: str, weight_quant: str = "bf16", name: str | None = None) -> tuple[ModelConfig, LazyCheckpoint]:
    """(config, lazy canonical view) of a checkpoint directory; `prepare_weights` reads it
    tensor by tensor and expert by expert (per-expert or fused expert tensors alike)."""
    with open(os.path.join(path, "config.json")) as f:
        d = json.load(f)
    cfg = config_from_hf(d, name or os.path.basename(os.path.normpath(path)), weight_quant)
    return cfg, LazyCheckpoint(path, cfg, bool(d.get("rope_interleave", True)))
