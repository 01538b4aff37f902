"""Tokenizers.  ``HFTokenizer`` wraps a ``tokenizer.json`` (the `tokenizers` library) when
a model directory provides one; ``ByteTokenizer`` is the self-contained fallback used with
synthetic weights: ids 0..2 are <pad>/<bos>/<eos>, ids 3..258 are the 256 byte values, and
larger ids (present in big vocabularies) decode to nothing."""
from __future__ import annotations

import os


class ByteTokenizer:
    PAD, BOS, EOS = 0, 1, 2
    OFFSET = 3

    def __init__(self, vocab_size: int = 259):
        self.vocab_size = max(vocab_size, 259)
        self.eos_token_id = self.EOS
        self.bos_token_id = self.BOS

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.BOS] if add_bos else []) + ids

    def decode(self, ids) -> str:
        bs = bytes(i - self.OFFSET for i in ids if self.OFFSET <= i < self.OFFSET + 256)
        return bs.decode("utf-8", errors="replace")


class IncrementalDecoder:
    """Streams text from token ids without splitting multi-byte characters."""

    def __init__(self, tok):
        self.tok = tok
        self.ids: list[int] = []
        self.emitted = 0

    def push(self, ids) -> str:
        self.ids.extend(ids)
        text = self.tok.decode(self.ids)
        if text.endswith("�"):
            return ""
        out = text[self.emitted:]
        self.emitted = len(text)
        return out


class HFTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer
        self.tk = Tokenizer.from_file(path)
        self.vocab_size = self.tk.get_vocab_size()
        self.eos_token_id = None
        self.bos_token_id = None
        for name in ("<|endoftext|>", "</s>", "<|im_end|>", "<｜end▁of▁sentence｜>"):
            i = self.tk.token_to_id(name)
            if i is not None:
                self.eos_token_id = i
                break

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        return self.tk.encode(text, add_special_tokens=add_bos).ids

    def decode(self, ids) -> str:
        return self.tk.decode(list(ids))


def load_tokenizer(model_dir: str | None, vocab_size: int):
    if model_dir:
        p = os.path.join(model_dir, "tokenizer.json")
        if os.path.exists(p):
            return HFTokenizer(p)
    return ByteTokenizer(vocab_size)
