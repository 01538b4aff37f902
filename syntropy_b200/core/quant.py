"""Quantisation schemes (reference: crates/core/src/quant.rs; plan/rfcs/RFC-0042 §1-§2)."""
from __future__ import annotations

import enum
from dataclasses import dataclass


class QuantKind(enum.Enum):
    PLAIN = "plain"          # f32 / f16 / bf16
    Q4_BLOCK = "q4"          # 32-element blocks, fp16 scale + min (GGUF Q4_1 interchange)
    FP8_BLOCK = "fp8"        # e4m3 with one f32 scale per 128x128 weight tile
    Q8_0 = "q8_0"


@dataclass(frozen=True)
class QuantScheme:
    kind: QuantKind
    block: tuple = ()
    dtype: str = "bf16"

    @property
    def bits_per_weight(self) -> float:
        if self.kind == QuantKind.Q4_BLOCK:
            return 5.0
        if self.kind == QuantKind.FP8_BLOCK:
            return 8.0 + 32.0 / (self.block[0] * self.block[1])
        if self.kind == QuantKind.Q8_0:
            return 8.5
        return {"f32": 32.0, "f16": 16.0, "bf16": 16.0}[self.dtype]

    @staticmethod
    def parse(s: str) -> "QuantScheme":
        s = s.lower()
        if s in ("q4", "q4_1", "q4_block"):
            return QuantScheme(QuantKind.Q4_BLOCK, (32,))
        if s in ("fp8", "fp8_block", "e4m3"):
            return QuantScheme(QuantKind.FP8_BLOCK, (128, 128))
        if s == "q8_0":
            return QuantScheme(QuantKind.Q8_0, (32,))
        if s in ("bf16", "f16", "f32", "fp32"):
            return QuantScheme(QuantKind.PLAIN, (), "f32" if s == "fp32" else s)
        raise ValueError(f"unknown quantisation scheme {s!r}")
