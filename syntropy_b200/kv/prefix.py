"""Prefix cache over full KV pages.

Each full page (block_size tokens) is named by a chained hash: h_i = H(h_{i-1}, tokens of
page i), so a page is reusable only after exactly the same token history.  Matching a new
prompt walks its full pages through the table and shares the hits (refcount); finished
sequences publish their full pages; the cache holds one reference per page and evicts the
least recently used unreferenced pages when the allocator runs low.
Reference: plan/rfcs/RFC-0022-kv-cache-prefix-cache-and-sessions.md :17, :355-365 (chained
page hashes with BLAKE3; the native BLAKE3 of csrc/cpu/blake3.cpp here).
"""
from __future__ import annotations

import struct
from collections import OrderedDict

from .._ext import ext
from .paged import BlockAllocator


def page_hash(parent: bytes, tokens) -> bytes:
    """BLAKE3(parent digest || tokens as u32 little-endian): 32 bytes."""
    return ext().blake3(parent + struct.pack(f"<{len(tokens)}I", *(int(t) for t in tokens)))


class PrefixCache:
    def __init__(self, alloc: BlockAllocator, block_size: int = 16, max_pages: int | None = None):
        self.alloc = alloc
        self.bs = block_size
        self.table: OrderedDict[bytes, int] = OrderedDict()  # hash -> block (LRU order)
        self.max_pages = max_pages
        self.hits = 0
        self.queries = 0

    def match(self, tokens: list[int]) -> tuple[list[int], int]:
        """Longest cached prefix of whole pages (leaving at least one token to compute).
        Returns (shared blocks, tokens covered); the blocks are increfed for the caller."""
        self.queries += 1
        blocks, parent = [], b""
        n_full = (len(tokens) - 1) // self.bs
        for i in range(n_full):
            h = page_hash(parent, tokens[i * self.bs:(i + 1) * self.bs])
            b = self.table.get(h)
            if b is None:
                break
            self.table.move_to_end(h)
            self.alloc.incref(b)
            blocks.append(b)
            parent = h
        if blocks:
            self.hits += 1
        return blocks, len(blocks) * self.bs

    def insert(self, tokens: list[int], blocks: list[int]):
        """Publish the full pages of a sequence (its KV for tokens[:len] is in `blocks`)."""
        parent = b""
        for i in range(min(len(tokens) // self.bs, len(blocks))):
            h = page_hash(parent, tokens[i * self.bs:(i + 1) * self.bs])
            if h not in self.table:
                self.alloc.incref(blocks[i])
                self.table[h] = blocks[i]
            else:
                self.table.move_to_end(h)
            parent = h
        if self.max_pages is not None:
            while len(self.table) > self.max_pages and self.evict(1):
                pass

    def evict(self, n: int) -> int:
        """Drop up to n least-recently-used pages that only the cache references."""
        freed = 0
        for h in list(self.table.keys()):
            if freed >= n:
                break
            b = self.table[h]
            if self.alloc.refcount[b] == 1:
                del self.table[h]
                self.alloc.free(b)
                freed += 1
        return freed

    @property
    def size(self) -> int:
        return len(self.table)
