"""Where preempted sequences' KV pages wait: host RAM up to a byte budget, then files.

When the VRAM page pool cannot hold the next decode step the engine preempts the newest
sequences: their pages are packed per layer on the device and copied to host memory
(`LLMEngine._swap_out`).  `SwapStore` keeps those packed layers in host RAM while their total
stays within `host_budget` bytes; a sequence preempted beyond that goes to a file in
`spill_dir` (an NVMe volume, typically) as a pack: 4 KiB-aligned extents with a JSON sidecar
and a BLAKE3 digest per extent, read back through the native pread pool (O_DIRECT when
aligned) and verified before the pages return to the device.  Sequences resume oldest first,
so the RAM tier holds the front of the queue and the file tier its tail; when a sequence
resumes, the next ones waiting on disk are read back into RAM as far as the budget allows.

Reference: plan/rfcs/RFC-0022-kv-cache-prefix-cache-and-sessions.md (VRAM -> host RAM -> NVMe
page tiers) and RFC-0041 §5 (packs: aligned extents plus a sidecar, verified by digest).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch


@dataclass
class SwapEntry:
    key: int
    nbytes: int
    layers: list | None = None       # host tensors while in RAM
    path: str | None = None          # pack file while on disk
    shapes: list = field(default_factory=list)
    dtype: torch.dtype = torch.bfloat16


class SwapStore:
    """Two tiers below VRAM for packed KV layers.  host_budget None: RAM only, unbounded;
    spill_dir None: no file tier (RAM grows past the budget rather than failing)."""

    def __init__(self, host_budget: int | None = None, spill_dir: str | None = None, io_threads: int = 4):
        if host_budget is not None and host_budget < 0:
            raise ValueError("host_budget: bytes >= 0")
        self.host_budget = host_budget
        self.spill_dir = spill_dir
        self.io_threads = io_threads
        if spill_dir is not None:
            os.makedirs(spill_dir, exist_ok=True)
        self.host_bytes = 0
        self.disk_bytes = 0
        self.stats = {"spilled": 0, "restored": 0, "spill_bytes": 0, "read_bytes": 0}

    # ------------------------------------------------------------------ tiers
    def _fits(self, n: int) -> bool:
        return self.host_budget is None or self.host_bytes + n <= self.host_budget

    def _spill(self, e: SwapEntry):
        from ..store.pack import write_pack
        # unique per process and store: several engines may share one spill directory
        path = os.path.join(self.spill_dir, f"kv_{os.getpid()}_{id(self):x}_{e.key}.pack")
        write_pack(path, {f"l{i}": t for i, t in enumerate(e.layers)})
        self.host_bytes -= e.nbytes
        self.disk_bytes += e.nbytes
        e.layers, e.path = None, path
        self.stats["spilled"] += 1
        self.stats["spill_bytes"] += e.nbytes

    def _load(self, e: SwapEntry):
        from ..store.pack import read_pack_into
        layers = [torch.empty(s, dtype=e.dtype) for s in e.shapes]
        got = read_pack_into(e.path, {f"l{i}": t for i, t in enumerate(layers)}, threads=self.io_threads)
        if got != e.nbytes:
            raise OSError(f"{e.path}: read {got} of {e.nbytes} bytes")
        self._remove_file(e)
        e.layers = layers
        self.host_bytes += e.nbytes
        self.stats["restored"] += 1
        self.stats["read_bytes"] += e.nbytes

    def _remove_file(self, e: SwapEntry):
        for p in (e.path, e.path + ".json"):
            try:
                os.remove(p)
            except FileNotFoundError:
                pass
        self.disk_bytes -= e.nbytes
        e.path = None

    # ------------------------------------------------------------------ API
    def put(self, key: int, layers: list) -> SwapEntry:
        """Stores a preempted sequence's packed layers (host tensors, one per layer)."""
        n = sum(t.numel() * t.element_size() for t in layers)
        e = SwapEntry(key, n, layers=layers, shapes=[tuple(t.shape) for t in layers],
                      dtype=layers[0].dtype if layers else torch.bfloat16)
        self.host_bytes += n
        if not self._fits(0) and self.spill_dir is not None:
            try:
                self._spill(e)
            except OSError:
                self.host_bytes -= n  # nothing was stored: the caller keeps the pages
                raise
        return e

    def take(self, e: SwapEntry) -> list:
        """The entry's layers in host memory (read back from its file if it was spilled); the
        entry leaves the store."""
        if e.layers is None:
            self._load(e)
        layers = e.layers
        e.layers = None
        self.host_bytes -= e.nbytes
        return layers

    def drop(self, e: SwapEntry):
        """Forgets an entry (its sequence was cancelled)."""
        if e.layers is not None:
            self.host_bytes -= e.nbytes
            e.layers = None
        if e.path is not None:
            self._remove_file(e)

    def refill(self, queue):
        """Reads spilled entries at the front of `queue` (entries in resume order) back into RAM
        while they fit the budget."""
        for e in queue:
            if e.layers is not None:
                continue
            if not self._fits(e.nbytes):
                break
            self._load(e)

    def where(self, e: SwapEntry) -> str:
        return "host" if e.layers is not None else "disk"
