"""Numerics contract of the kernels: tolerance tables, an accumulation-precision detector, and
per-op provider selection.

* `TOLERANCES`: the relative error (||got - want|| / ||want||, against the f32 reference of the
  same op on the same dequantised operands) each dtype class may show.  Versioned: a kernel
  change that needs a looser bound bumps `TOLERANCE_VERSION`.
* `accumulation_class(fn)`: feeds a dot product whose terms vanish when added one by one in a
  16-bit accumulator (1 followed by many tiny terms whose sum is large) and reports the
  accumulator class the kernel shows: "f32" or "reduced".
* `Selector`: chooses among providers of one op for one shape signature.  Every candidate
  must first pass its certificate (the tolerance table against the f32 reference on a probe
  input); certified candidates are then timed, and a candidate replaces the default only when
  it is faster by more than `margin` (3%).  Decisions are cached per (op, shape) and can be
  saved and loaded.

Reference: crates/kernels/src/select.rs:199-668 (certificates, microbenchmark, 3% margin),
crates/kernels/src/tolerances.rs and numerics/tolerances-v1.toml (per-class tables),
crates/kernels/src/numerics.rs:317-435 (reduced-precision accumulation detector).
"""
from __future__ import annotations

import json
import time
from dataclasses import dataclass, field

import torch

TOLERANCE_VERSION = 1
# relative-norm bounds against the f32 reference on the same (dequantised) operands
TOLERANCES = {
    "f32": 1e-5,          # f32 operands, f32 accumulation
    "bf16_out": 1e-2,     # bf16 outputs (one rounding of each element)
    "bf16_f32acc": 1e-4,  # bf16 operands, f32 accumulation, f32 outputs
    "q4_f32acc": 1e-4,    # 4-bit weights dequantised exactly, f32 accumulation, f32 outputs
    "fp8_act": 6e-2,      # e4m3 activations (quantised per 1x128 block)
    "int8_act": 1e-2,     # int8 activations (quantised per 32-element block)
}


def rel_err(got: torch.Tensor, want: torch.Tensor) -> float:
    return ((got.float() - want.float()).norm() / want.float().norm().clamp_min(1e-30)).item()


def within(cls: str, got: torch.Tensor, want: torch.Tensor) -> bool:
    return rel_err(got, want) <= TOLERANCES[cls]


def accumulation_class(dot, n: int = 4096, device="cpu") -> str:
    """dot(x [1, n] bf16, w [1, n] bf16) -> [1] float: one product of 1 then n - 1 products of
    2^-10 (exact in bf16; each below half an ulp of 1 in bf16, so a 16-bit accumulator that adds
    them one by one keeps 1, an f32 one reaches 1 + (n - 1) / 1024)."""
    x = torch.full((1, n), 2.0 ** -10, dtype=torch.bfloat16, device=device)
    x[0, 0] = 1.0
    w = torch.ones(1, n, dtype=torch.bfloat16, device=device)
    got = float(dot(x, w).reshape(-1)[0])
    want = 1.0 + (n - 1) * 2.0 ** -10
    return "f32" if abs(got - want) <= 1e-3 * want else "reduced"


@dataclass
class Candidate:
    name: str
    fn: object            # fn(*inputs) -> output
    dtype_class: str      # tolerance class of its output


@dataclass
class Selector:
    margin: float = 0.03
    iters: int = 10
    timer: object = None  # timer(name, fn) -> seconds per call (default: CUDA events or wall clock)
    decisions: dict = field(default_factory=dict)
    log: list = field(default_factory=list)

    def _time(self, name, fn) -> float:
        if self.timer is not None:
            return self.timer(name, fn)
        if torch.cuda.is_available():
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(self.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / 1e3 / self.iters
        fn()
        t0 = time.perf_counter()
        for _ in range(self.iters):
            fn()
        return (time.perf_counter() - t0) / self.iters

    def choose(self, op: str, shape: tuple, candidates: list[Candidate], inputs: tuple, reference) -> str:
        """Name of the provider for (op, shape): candidates[0] is the default.  reference(*inputs)
        is the f32 result the certificates compare with."""
        key = f"{op}:{'x'.join(map(str, shape))}"
        if key in self.decisions:
            return self.decisions[key]
        want = reference(*inputs)
        certified, times = [], {}
        for c in candidates:
            try:
                ok = within(c.dtype_class, c.fn(*inputs), want)
            except Exception as e:  # noqa: BLE001  (a provider that cannot run this shape)
                self.log.append({"key": key, "candidate": c.name, "certified": False, "error": str(e)[:200]})
                continue
            self.log.append({"key": key, "candidate": c.name, "certified": ok})
            if ok:
                certified.append(c)
        if not certified:
            raise RuntimeError(f"{key}: no provider passed its certificate")
        for c in certified:
            times[c.name] = self._time(c.name, lambda c=c: c.fn(*inputs))
        pick = certified[0].name
        for c in certified[1:]:
            if times[c.name] < times[pick] * (1.0 - self.margin):
                pick = c.name
        self.decisions[key] = pick
        self.log.append({"key": key, "times_us": {k: round(v * 1e6, 2) for k, v in times.items()}, "pick": pick})
        return pick

    def save(self, path: str):
        with open(path, "w") as f:
            json.dump({"version": TOLERANCE_VERSION, "decisions": self.decisions}, f, indent=1)

    def load(self, path: str):
        with open(path) as f:
            d = json.load(f)
        if d.get("version") == TOLERANCE_VERSION:
            self.decisions.update(d["decisions"])
