"""Configuration schema as dataclasses and its layered resolution.

defaults < TOML file < `SYN_<SECTION>_<KEY>` environment < CLI `section.key=value`, with the
origin of every value kept (a file value as `file path:line`), so errors name where the bad
value came from.  Typed values: sizes ("64GiB", "512MB", plain bytes) and durations ("250ms",
"2s", "1m", plain seconds) for the fields marked with a unit.
Reference: crates/config/src/{registry.rs,resolve.rs,validate.rs,origin.rs} (schema as code,
layered resolution, file:line diagnostics, value types).
"""
from __future__ import annotations

import dataclasses
import os
import re
from dataclasses import dataclass, field, fields

_SIZE = {"": 1, "b": 1, "kb": 10**3, "mb": 10**6, "gb": 10**9, "tb": 10**12,
         "kib": 2**10, "mib": 2**20, "gib": 2**30, "tib": 2**40}
_TIME = {"": 1.0, "s": 1.0, "ms": 1e-3, "us": 1e-6, "m": 60.0, "h": 3600.0}


def parse_size(v) -> int:
    """'64GiB' / '512 MB' / 1024 -> bytes."""
    if isinstance(v, (int, float)) and not isinstance(v, bool):
        return int(v)
    m = re.fullmatch(r"\s*([0-9]*\.?[0-9]+)\s*([a-zA-Z]*)\s*", str(v))
    if not m or m.group(2).lower() not in _SIZE:
        raise ValueError(f"not a size: {v!r}")
    return int(float(m.group(1)) * _SIZE[m.group(2).lower()])


def parse_duration(v) -> float:
    """'250ms' / '2s' / '1m' / 0.5 -> seconds."""
    if isinstance(v, (int, float)) and not isinstance(v, bool):
        return float(v)
    m = re.fullmatch(r"\s*([0-9]*\.?[0-9]+)\s*([a-zA-Z]*)\s*", str(v))
    if not m or m.group(2).lower() not in _TIME:
        raise ValueError(f"not a duration: {v!r}")
    return float(m.group(1)) * _TIME[m.group(2).lower()]


def _size(default):
    return field(default=default, metadata={"unit": "size"})


def _dur(default):
    return field(default=default, metadata={"unit": "duration"})

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
    peer_timeout_s: float = _dur(2.0)  # bounded device waits on peer flags


@dataclass
class SchedSection:
    max_batch: int = 64
    max_prefill_tokens: int = 8192
    cuda_graphs: bool = True
    chunk_tokens: int = 0            # chunked prefill with decode-first steps (0 = whole prompts)


@dataclass
class TierSection:
    expert_cache_frac: float = 1.0   # VRAM-resident share of each rank's experts
    kv_budget: int = _size(0)        # KV cache bytes; 0 = sized from max_batch x max_seq_len
    rebalance_every: int = 64        # decode steps between expert-cache rebalances
    expert_prefetch: bool = True     # router-predicted prefetch of host experts during decode
    cpu_expert_share: float = 0.0    # share of each layer's host experts computed by host threads
    cpu_threads: int = 0             # 0 = every allowed core but two
    kv_host_budget: int = _size(0)   # host RAM for preempted sequences' KV pages; 0 = unbounded
    kv_spill_dir: str = ""           # pack files for preempted KV past kv_host_budget ("" = none)


@dataclass
class KernelsSection:
    deterministic: bool = True           # fixed reduction orders everywhere (the only mode built)
    spin_timeout: float = _dur(2.0)      # limit of every device-side wait (doorbells, peers, CPU tier)
    cpu_gemv_mode: int = -1              # CPU expert kernels: -1 default, 0 C++, 1 AVX-512 BF16, 2 VNNI


@dataclass
class SpecSection:
    drafter: str = "none"        # none | ngram | mtp | draft
    gamma: int = 2               # drafted tokens per verify window
    draft_model: str = ""        # preset name of the draft model (drafter = draft)
    draft_temperature: float = 0.0  # > 0: drafts sampled from the draft model (stochastic-draft acceptance)


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
    # kill switches, each falling back to a plainer path that stays correct: cuda_graph (eager
    # decode steps), expert_prefetch (host experts read in place), cpu_tier (no host CPU experts),
    # speculative (plain decode), tcgen05_attention (the mma.sync prefill attention kernel),
    # tcgen05_bf16_gemm (the library GEMM for bf16 weights)
    disable: list = field(default_factory=list)


FEATURES = ("cuda_graph", "expert_prefetch", "cpu_tier", "speculative", "tcgen05_attention", "tcgen05_bf16_gemm")


@dataclass
class Config:
    model: ModelSection = field(default_factory=ModelSection)
    parallel: ParallelSection = field(default_factory=ParallelSection)
    sched: SchedSection = field(default_factory=SchedSection)
    tier: TierSection = field(default_factory=TierSection)
    api: ApiSection = field(default_factory=ApiSection)
    kernels: KernelsSection = field(default_factory=KernelsSection)
    spec: SpecSection = field(default_factory=SpecSection)
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
        unit = names[key].metadata.get("unit")
        try:
            if unit == "size":
                val = parse_size(raw)
            elif unit == "duration":
                val = parse_duration(raw)
            else:
                val = _coerce(raw, cur, dotted, origin)
        except ValueError as e:
            raise ValueError(f"{dotted}: {e} ({origin})") from None
        setattr(obj, key, val)
        self.origin[dotted] = origin

    def validate(self):
        errs = []

        def err(key, msg):
            errs.append(f"{key} {msg} ({self.origin.get(key, 'default')})")

        for key in ("tier.expert_cache_frac", "tier.cpu_expert_share"):
            sec, _, k = key.partition(".")
            if not 0.0 <= getattr(getattr(self, sec), k) <= 1.0:
                err(key, "must be in [0, 1]")
        for k in ("tp", "ep", "pp"):
            v = getattr(self.parallel, k)
            if v < 1 or v & (v - 1):
                err(f"parallel.{k}", "must be a power of two >= 1")
        if self.sched.max_batch < 1:
            err("sched.max_batch", "must be >= 1")
        if self.sched.chunk_tokens < 0:
            err("sched.chunk_tokens", "must be >= 0")
        unknown = [f for f in self.features.disable if f not in FEATURES]
        if unknown:
            err("features.disable", f"names unknown switches {unknown} (known: {', '.join(FEATURES)})")
        if self.spec.drafter not in ("none", "ngram", "mtp", "draft"):
            err("spec.drafter", "must be one of none, ngram, mtp, draft")
        if self.spec.drafter == "draft" and not self.spec.draft_model:
            err("spec.draft_model", "is required with spec.drafter = draft")
        if self.spec.gamma < 1:
            err("spec.gamma", "must be >= 1")
        if self.kernels.cpu_gemv_mode not in (-1, 0, 1, 2):
            err("kernels.cpu_gemv_mode", "must be -1, 0, 1 or 2")
        if not 0.0 < self.kernels.spin_timeout <= 60.0:
            err("kernels.spin_timeout", "must be in (0, 60] seconds")
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


def _line_of(lines: list[str], section: str | None, key: str) -> int:
    """1-based line of `key = ...` inside `[section]` (0 if not found)."""
    cur = None
    for i, ln in enumerate(lines, 1):
        t = ln.strip()
        m = re.fullmatch(r"\[\s*([^\]]+?)\s*\]", t)
        if m:
            cur = m.group(1)
            if section is None and cur == key:
                return i
            continue
        if cur == section and re.match(rf"{re.escape(key)}\s*=", t):
            return i
    return 0


def load_config(path: str | None = None, env: dict | None = None, overrides: list[str] | None = None) -> Config:
    """defaults < file < env < CLI overrides ("section.key=value")."""
    cfg = Config()
    if path:
        if tomllib is None:
            raise RuntimeError("tomllib unavailable")
        with open(path, "rb") as f:
            raw = f.read()
        data = tomllib.loads(raw.decode())
        lines = raw.decode().splitlines()
        for sec, vals in data.items():
            if not isinstance(vals, dict):
                raise KeyError(f"{path}:{_line_of(lines, None, sec)}: top-level key {sec!r} is not a section")
            for k, v in vals.items():
                cfg.set(f"{sec}.{k}", v, f"file {path}:{_line_of(lines, sec, k)}")
    env = os.environ if env is None else env
    for k, v in env.items():
        if not k.startswith("SYN_"):
            continue
        rest = k[4:].lower()
        sec, _, key = rest.partition("_")
        if sec in ("model", "parallel", "sched", "tier", "api", "kernels", "spec", "debug", "features") and key:
            cfg.set(f"{sec}.{key}", v, f"env {k}")
    for o in overrides or []:
        k, _, v = o.partition("=")
        cfg.set(k.strip(), v.strip(), f"cli {o}")
    return cfg.validate()
