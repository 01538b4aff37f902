"""Tokenizers and chat templates (reference: crates/text)."""
from .tokenizer import ByteTokenizer, HFTokenizer, load_tokenizer  # noqa: F401
from .chat import apply_chat_template  # noqa: F401
