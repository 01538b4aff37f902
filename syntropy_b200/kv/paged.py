"""Paged KV cache with fixed-size token pages (16 tokens by default).

Device layout is layer-first: per layer K and V tensors of shape
[num_blocks, n_kv_heads, block_size, head_dim], so one page of one KV head is a
contiguous 4 KB run for head_dim 128 in bf16 (the decode kernel's cp.async unit).
Reference design: plan/rfcs/RFC-0022-kv-cache-prefix-cache-and-sessions.md §2-§4 (page
classes, layer-first device layout, page-first host layout).

Block 0 is reserved as the null page that padded rows of a captured batch read.
"""
from __future__ import annotations

import torch


class BlockAllocator:
    """Free list of page ids with reference counts (shared prefix pages)."""

    def __init__(self, num_blocks: int, reserved: int = 1):
        self.num_blocks = num_blocks
        self.reserved = reserved
        self._free = list(range(num_blocks - 1, reserved - 1, -1))
        self.refcount = [0] * num_blocks

    @property
    def num_free(self) -> int:
        return len(self._free)

    def alloc(self) -> int:
        if not self._free:
            raise MemoryError("KV cache out of pages")
        b = self._free.pop()
        self.refcount[b] = 1
        return b

    def incref(self, b: int):
        self.refcount[b] += 1

    def free(self, b: int):
        self.refcount[b] -= 1
        if self.refcount[b] == 0:
            self._free.append(b)


class PagedKVCache:
    def __init__(self, n_layers: int, num_blocks: int, n_kv_heads: int, head_dim: int, block_size: int = 16,
                 dtype=torch.bfloat16, device="cpu", with_v: bool = True):
        self.n_layers = n_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        shape = (num_blocks, n_kv_heads, block_size, head_dim)
        self.k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(n_layers)]
        # latent caches (MLA) keep one tensor per layer: V aliases K
        self.v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(n_layers)] if with_v else self.k
        self.alloc = BlockAllocator(num_blocks)

    @staticmethod
    def bytes_per_block(n_layers, n_kv_heads, head_dim, block_size=16, dtype_bytes=2) -> int:
        return 2 * n_layers * n_kv_heads * block_size * head_dim * dtype_bytes

    def blocks_needed(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size

    def ensure(self, blocks: list[int], n_tokens: int) -> list[int]:
        """Grow a sequence's block list to hold ``n_tokens`` tokens."""
        while len(blocks) < self.blocks_needed(n_tokens):
            blocks.append(self.alloc.alloc())
        return blocks

    def release(self, blocks: list[int]):
        for b in blocks:
            self.alloc.free(b)
        blocks.clear()

    def slot(self, blocks: list[int], pos: int) -> int:
        return blocks[pos // self.block_size] * self.block_size + pos % self.block_size
