"""Grammar-constrained decoding: the vocabulary as byte strings, constraint construction and
logit masking.  The automata and the vocabulary trie are native (``csrc/cpu/constrain.cpp``).

Constraints (``SamplingParams.constraint``):

* ``{"type": "json"}`` — the output is one JSON text whose top-level value is an object
  (OpenAI ``response_format: {"type": "json_object"}``); the sequence stops when it closes;
* ``{"choices": ["yes", "no", ...]}`` — the output is exactly one of the strings.

Reference: crates/text/src/constraint/{engine.rs,llg.rs,schema.rs} (token masks from a grammar
with a vocabulary cache).
"""
from __future__ import annotations

import torch

from .._ext import ext


def _gpt2_byte_decoder() -> dict[str, int]:
    """Inverse of the byte-level BPE alphabet: printable Latin-1 bytes stand for themselves, the
    other bytes are mapped in order onto code points 256, 257, ... (the public GPT-2 scheme)."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[chr(b)] = b
        else:
            table[chr(256 + extra)] = b
            extra += 1
    return table


def vocab_bytes(tokenizer, vocab_size: int) -> list[bytes]:
    """Byte string of every token id (b"" for special tokens and ids the tokenizer lacks)."""
    from .tokenizer import ByteTokenizer
    out = [b""] * vocab_size
    if tokenizer is None or isinstance(tokenizer, ByteTokenizer):
        off = ByteTokenizer.OFFSET
        for b in range(256):
            if off + b < vocab_size:
                out[off + b] = bytes([b])
        return out
    tk = tokenizer.tk
    vocab = tk.get_vocab(with_added_tokens=False)
    special = set(tk.get_vocab(with_added_tokens=True)) - set(vocab)
    byte_level = any("Ġ" in t or "Ċ" in t for t in list(vocab)[:5000])
    dec = _gpt2_byte_decoder() if byte_level else None
    for tok, i in vocab.items():
        if i >= vocab_size or tok in special:
            continue
        if dec is not None:
            try:
                out[i] = bytes(dec[ch] for ch in tok)
            except KeyError:
                out[i] = tok.encode("utf-8")
        elif len(tok) == 6 and tok.startswith("<0x") and tok.endswith(">"):
            out[i] = bytes([int(tok[3:5], 16)])  # sentencepiece byte fallback
        else:
            out[i] = tok.replace("▁", " ").encode("utf-8")
    return out


def make_constraint(trie, eos: int | None, spec):
    """Native constraint for a request's spec (see the module docstring)."""
    e = -1 if eos is None else int(eos)
    if isinstance(spec, str):
        spec = {"type": spec}
    if spec.get("choices") is not None:
        opts = [c.encode("utf-8") if isinstance(c, str) else bytes(c) for c in spec["choices"]]
        return ext().Constraint.choices(trie, e, opts)
    if spec.get("type") in ("json", "json_object", "json_schema"):
        return ext().Constraint.json(trie, e)
    raise ValueError(f"unknown constraint {spec!r}")


def allowed(mask_words: torch.Tensor, vocab: int) -> torch.Tensor:
    """int32 bitmask words -> bool [vocab]."""
    bits = (mask_words.view(-1, 1) >> torch.arange(32, dtype=torch.int32)) & 1
    return bits.reshape(-1)[:vocab].bool()


def mask_logits(logits: torch.Tensor, constraints) -> torch.Tensor:
    """Copy of logits [n, V] with every token a row's constraint forbids at -inf."""
    out = logits.clone()
    V = logits.shape[1]
    for i, c in enumerate(constraints):
        ok = allowed(c.mask(), V).to(logits.device)
        out[i].masked_fill_(~ok, float("-inf"))
    return out
