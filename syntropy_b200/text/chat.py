"""Chat templates: ChatML-style turns (the Qwen family's format) with a generic fallback."""
from __future__ import annotations


def apply_chat_template(messages: list[dict], system: str | None = None, add_generation_prompt: bool = True) -> str:
    parts = []
    if system:
        parts.append(f"<|im_start|>system\n{system}<|im_end|>\n")
    for m in messages:
        content = m.get("content", "")
        if isinstance(content, list):  # OpenAI/Anthropic content blocks
            content = "".join(b.get("text", "") for b in content if isinstance(b, dict))
        parts.append(f"<|im_start|>{m.get('role', 'user')}\n{content}<|im_end|>\n")
    if add_generation_prompt:
        parts.append("<|im_start|>assistant\n")
    return "".join(parts)


def chat_ids(tokenizer, msgs: list[dict], system: str | None = None) -> list[int]:
    """Chat prompt ids: span-aware encoding where the tokenizer has it (message content cannot
    inject special tokens), else the tokenizer's own chat template (checkpoint directories) or
    ChatML, encoded as text."""
    if hasattr(tokenizer, "encode_chat"):
        return tokenizer.encode_chat(msgs, system)
    tmpl = getattr(tokenizer, "apply_chat_template", apply_chat_template)
    return tokenizer.encode(tmpl(msgs, system=system) if system else tmpl(msgs))
