"""Tokenizers.  ``HFTokenizer`` wraps a ``tokenizer.json`` (the `tokenizers` library) when
a model directory provides one; ``ByteTokenizer`` is the self-contained fallback used with
synthetic weights: ids 0..2 are <pad>/<bos>/<eos>, ids 3..258 are the 256 byte values, and
larger ids (present in big vocabularies) decode to nothing."""
from __future__ import annotations

import os
import re


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
    """`tokenizer.json` through the `tokenizers` library, plus what a checkpoint directory says
    about it: the chat template (Jinja, `tokenizer_config.json`), BOS/EOS tokens and the stop
    ids of `generation_config.json` (a list: chat models stop on end-of-turn too)."""

    def __init__(self, path: str):
        from tokenizers import Tokenizer
        self.tk = Tokenizer.from_file(path)
        self.vocab_size = self.tk.get_vocab_size()
        d = os.path.dirname(path)
        conf = _read_json(os.path.join(d, "tokenizer_config.json"))
        gen = _read_json(os.path.join(d, "generation_config.json"))
        self.chat_template = conf.get("chat_template")
        if isinstance(self.chat_template, list):  # named templates: take the default one
            self.chat_template = next((t["template"] for t in self.chat_template if t.get("name") == "default"),
                                      self.chat_template[0]["template"])
        self.bos_token = _tok_str(conf.get("bos_token"))
        self.eos_token = _tok_str(conf.get("eos_token"))
        self.bos_token_id = self.tk.token_to_id(self.bos_token) if self.bos_token else None
        stop = gen.get("eos_token_id")
        stop = stop if isinstance(stop, list) else ([stop] if stop is not None else [])
        if self.eos_token and self.tk.token_to_id(self.eos_token) is not None:
            stop = [self.tk.token_to_id(self.eos_token)] + [i for i in stop if i != self.tk.token_to_id(self.eos_token)]
        if not stop:
            for name in ("<|endoftext|>", "</s>", "<|im_end|>", "<｜end▁of▁sentence｜>"):
                i = self.tk.token_to_id(name)
                if i is not None:
                    stop = [i]
                    break
        self.stop_token_ids = stop
        self.eos_token_id = stop[0] if stop else None

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        return self.tk.encode(text, add_special_tokens=add_bos).ids

    def decode(self, ids) -> str:
        return self.tk.decode(list(ids))

    def encode_literal(self, text: str) -> list[int]:
        """Text as plain text: special-token strings inside it stay text."""
        self.tk.encode_special_tokens = True
        try:
            return self.tk.encode(text, add_special_tokens=False).ids
        finally:
            self.tk.encode_special_tokens = False

    def encode_chat(self, messages: list[dict], system: str | None = None,
                    add_generation_prompt: bool = True) -> list[int]:
        """Token ids of a chat with span-aware encoding (the injection guard of reference
        crates/text/src/tokenizer/spans.rs): the template's own text may produce special
        tokens, message content is encoded literally, so a user who types "<|im_end|>" gets
        those characters, not the end-of-turn token.  Spans are encoded one by one, which
        gives the ids of the whole rendered prompt for tokenizers whose pre-tokenizer splits
        at those boundaries anyway and adds no prefix space (Llama 3, Qwen)."""
        marks = [f"\x00\x01span{i}\x01\x00" for i in range(len(messages) + 1)]
        sys_mark = marks[-1] if system else None
        masked = [dict(m, content=marks[i]) for i, m in enumerate(messages)]
        text = self.apply_chat_template(masked, sys_mark, add_generation_prompt)
        trim = bool(self.chat_template) and "trim" in self.chat_template  # the template strips content
        spans = {marks[i]: (_text(m.get("content", "")).strip() if trim else _text(m.get("content", "")))
                 for i, m in enumerate(messages)}
        if system:
            spans[sys_mark] = system
        ids, pos = [], 0
        pattern = re.compile("|".join(re.escape(k) for k in spans))
        for mt in pattern.finditer(text):
            if mt.start() > pos:
                ids += self.tk.encode(text[pos:mt.start()], add_special_tokens=False).ids
            ids += self.encode_literal(spans[mt.group(0)])
            pos = mt.end()
        if pos < len(text):
            ids += self.tk.encode(text[pos:], add_special_tokens=False).ids
        return ids

    def apply_chat_template(self, messages: list[dict], system: str | None = None,
                            add_generation_prompt: bool = True) -> str:
        """The checkpoint's own template (sandboxed Jinja), else ChatML."""
        from .chat import apply_chat_template as chatml
        if not self.chat_template:
            return chatml(messages, system, add_generation_prompt)
        msgs = ([{"role": "system", "content": system}] if system else []) + [
            dict(m, content=_text(m.get("content", ""))) for m in messages]
        from jinja2.sandbox import ImmutableSandboxedEnvironment
        env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)

        def raise_exception(msg):
            raise ValueError(msg)
        env.globals["raise_exception"] = raise_exception
        return env.from_string(self.chat_template).render(
            messages=msgs, add_generation_prompt=add_generation_prompt, bos_token=self.bos_token or "",
            eos_token=self.eos_token or "")


def _read_json(p: str) -> dict:
    import json
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def _tok_str(v):
    return v.get("content") if isinstance(v, dict) else v


def _text(content) -> str:
    if isinstance(content, list):  # OpenAI / Anthropic content blocks
        return "".join(b.get("text", "") for b in content if isinstance(b, dict))
    return content


def load_tokenizer(model_dir: str | None, vocab_size: int):
    if model_dir:
        p = os.path.join(model_dir, "tokenizer.json")
        if os.path.exists(p):
            return HFTokenizer(p)
    return ByteTokenizer(vocab_size)
