"""Configuration schema as dataclasses and its layered resolution."""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field, fields

try:
    import tomllib
except ImportError:  # pragma: no cover
    tomllib = None


@dataclass
class ModelSection:
    name: str = "qwen3-235b-a22b"
    path: str = ""                 # directory with safetensors / GGUF files ("" = synthetic weights)
    quant: str = ""                # override the preset's weight quantisation
    seed: int = 0
    max_seq_len: int = 4096


@dataclass
class ParallelSection:
    tp: int = 1
    ep: int = 1
    pp: int = 1
    fused_collectives: bool = True  # False -> NCCL baseline data plane
    peer_timeout_s: float = 2.0     # bounded device waits on peer flags


@dataclass
class SchedSection:
    max_batch: int = 64
    max_prefill_tokens: int = 8192
    cuda_graphs: bool = True


@dataclass
class TierSection:
    expert_cache_frac: float = 1.0   # VRAM-resident share of each rank's experts
    kv_budget_gb: float = 0.0        # 0 = sized from max_batch x max_seq_len
    rebalance_every: int = 64        # decode steps between expert-cache rebalances


@dataclass
class ApiSection:
    host: str = "127.0.0.1"
    port: int = 8000
    model_id: str = "syntropy"
    max_body: int = 32 << 20


@dataclass
class DebugSection:
    bench_api: bool = True
    telemetry_api: bool = False


@dataclass
class FeaturesSection:
    disable: list = field(default_factory=list)  # kill switches: "cuda_graph", "fused_collectives", ...


@dataclass
class Config:
    model: ModelSection = field(default_factory=ModelSection)
    parallel: ParallelSection = field(default_factory=ParallelSection)
    sched: SchedSection = field(default_factory=SchedSection)
    tier: TierSection = field(default_factory=TierSection)
    api: ApiSection = field(default_factory=ApiSection)
    debug: DebugSection = field(default_factory=DebugSection)
    features: FeaturesSection = field(default_factory=FeaturesSection)
    origin: dict = field(default_factory=dict, repr=False)

    def feature(self, name: str) -> bool:
        return name not in self.features.disable

    def set(self, dotted: str, raw, origin: str):
        sec, _, key = dotted.partition(".")
        if not hasattr(self, sec) or sec == "origin":
            raise KeyError(f"unknown config section {sec!r} ({origin})")
        obj = getattr(self, sec)
        names = {f.name: f for f in fields(obj)}
        if key not in names:
            raise KeyError(f"unknown config key {dotted!r} ({origin})")
        cur = getattr(obj, key)
        setattr(obj, key, _coerce(raw, cur, dotted, origin))
        self.origin[dotted] = origin

    def validate(self):
        errs = []
        if not 0.0 <= self.tier.expert_cache_frac <= 1.0:
            errs.append(f"tier.expert_cache_frac must be in [0, 1] ({self.origin.get('tier.expert_cache_frac', 'default')})")
        for k in ("tp", "ep", "pp"):
            v = getattr(self.parallel, k)
            if v < 1 or v & (v - 1):
                errs.append(f"parallel.{k} must be a power of two >= 1")
        if self.sched.max_batch < 1:
            errs.append("sched.max_batch must be >= 1")
        if errs:
            raise ValueError("; ".join(errs))
        return self

    def to_dict(self) -> dict:
        d = dataclasses.asdict(self)
        d.pop("origin", None)
        return d


def _coerce(raw, cur, key, origin):
    if isinstance(raw, type(cur)) and not isinstance(cur, bool):
        return raw
    try:
        if isinstance(cur, bool):
            if isinstance(raw, bool):
                return raw
            s = str(raw).strip().lower()
            if s in ("1", "true", "yes", "on"):
                return True
            if s in ("0", "false", "no", "off"):
                return False
            raise ValueError(s)
        if isinstance(cur, int):
            return int(raw)
        if isinstance(cur, float):
            return float(raw)
        if isinstance(cur, list):
            return list(raw) if isinstance(raw, (list, tuple)) else [x for x in str(raw).split(",") if x]
        return str(raw)
    except ValueError as e:
        raise ValueError(f"{key}: cannot parse {raw!r} as {type(cur).__name__} ({origin})") from e


def load_config(path: str | None = None, env: dict | None = None, overrides: list[str] | None = None) -> Config:
    """defaults < file < env < CLI overrides ("section.key=value")."""
    cfg = Config()
    if path:
        if tomllib is None:
            raise RuntimeError("tomllib unavailable")
        with open(path, "rb") as f:
            data = tomllib.load(f)
        for sec, vals in data.items():
            if not isinstance(vals, dict):
                raise KeyError(f"{path}: top-level key {sec!r} is not a section")
            for k, v in vals.items():
                cfg.set(f"{sec}.{k}", v, f"file {path}")
    env = os.environ if env is None else env
    for k, v in env.items():
        if not k.startswith("SYN_"):
            continue
        rest = k[4:].lower()
        sec, _, key = rest.partition("_")
        if sec in ("model", "parallel", "sched", "tier", "api", "debug", "features") and key:
            cfg.set(f"{sec}.{key}", v, f"env {k}")
    for o in overrides or []:
        k, _, v = o.partition("=")
        cfg.set(k.strip(), v.strip(), f"cli {o}")
    return cfg.validate()
