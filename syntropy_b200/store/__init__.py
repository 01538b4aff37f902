"""Local model store: model directories indexed by content digest (reference: crates/store)."""
from .local import ModelStore  # noqa: F401
