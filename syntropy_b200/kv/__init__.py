"""Paged KV cache: block allocator, per-sequence block tables, prefix cache."""
from .paged import BlockAllocator, PagedKVCache  # noqa: F401
