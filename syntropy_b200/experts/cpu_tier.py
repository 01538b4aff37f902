"""Cold experts computed on the host CPU during decode, next to the PCIe path.

With a VRAM cap, every MoE layer has host experts.  The GPU can read them over PCIe in place
(the grouped GEMV takes host pointers), which is bound by the link (~50 GB/s).  The host's own
DRAM bandwidth is a second, independent resource: a share of the host experts
(``cpu_share``) is computed by a pool of CPU threads (AVX-512 int16 VNNI or BF16, whichever is
faster on the host, over the same tiled 4-bit rows, ``csrc/cpu/cpu_experts.cpp``) while the GPU streams the resident experts and the
remaining host experts.  Per MoE layer of a decode step:

1. routing on the GPU; ``cpu_handoff`` copies the layer's rows and routing CSR into a pinned
   mailbox and raises its go word;
2. the GPU runs its grouped GEMVs, which skip the CPU's experts (null weight pointers in the
   layer's tables); the CPU threads compute theirs at the same time;
3. ``cpu_collect`` waits for the done word (with a time limit: a missing CPU answer sets a
   status bit instead of hanging the GPU) and copies the CPU rows into the pair outputs;
4. the ordered combine runs as before.

All of it is captured in the decode CUDA graphs (the sequence number lives on the device).

Reference: crates/kernels-cpu/src/moe.rs (expert misses on the CPU), crates/kernels/src/moe/
doorbell.rs and split.rs (host-mapped doorbell, hit / miss / CPU sites).
"""
from __future__ import annotations

import os

import torch

from .._ext import ext


# Host-tier rates used to split each rank's cold experts between its CPU workers and its PCIe
# link (bytes of 4-bit weights per second), per CPU kernel family (`ext().cpu_gemv_mode()`, the
# faster of the two on the host, timed at start-up).  Measured on the B200 node (16-core Xeon
# slice, 14 workers, capped Qwen3 decode on one GPU): the int16 VNNI pool balances the link at a
# share of 0.7 (shares 0.6 / 0.7 / 0.75 / 0.8 gave 68.4 / 71.4 / 67.7 / 57.8 tok/s), i.e. ~7.5
# GB/s per worker; the BF16 pool at 0.6 (0.5 / 0.6 / 0.75 gave 57.3 / 65.4 / 55.8), ~4.8 GB/s per
# worker (its `vdpbf16ps` issues at about a quarter of the FMA rate on that host).  One GPU stages
# host rows with bulk DMA at ~45 GB/s while the CPU also streams DRAM.  With several ranks per
# node the workers of all ranks contend for DRAM while each GPU stages over its own link; the
# effective link rate that reproduces the measured balance is ~55 GB/s per GPU (capped Qwen3
# decode over EP2 with 11 BF16 workers per rank: shares 0.68 / 0.56 / 0.5 gave 71.7 / 78.1 /
# 90.1 tok/s).
CPU_GBS_PER_THREAD = {1: 4.8, 2: 7.5}
# With several ranks on a node the pools of all ranks share the host's DRAM: on the 2-GPU node
# slice (24 cores, 11 int16 workers per rank) a rank's pool reached ~57 GB/s at share 0.6
# (86.4 tok/s, 370 ms per step, the CPU part the longer one), below its 11 x 7.5 GB/s of
# instruction throughput, so the model caps a rank's pool there.
CPU_GBS_PER_RANK_SHARED = 57.0
PCIE_GBS_ALONE, PCIE_GBS_SHARED = 45.0, 55.0
# Eight ranks per node: GPU pairs share a host link; EP8 staged 7.76 GB per rank in 305 ms
# (~25 GB/s per rank) on the B200 node.  (Four ranks balanced at the EP2 rate: share 0.49 gave
# 93.2 tok/s against 88.1 / 90.0 at 0.62 / 0.75.)
PCIE_GBS_PAIRED = 25.0


def rank_cpus(local_rank: int, local_world: int, allowed: list[int] | None = None) -> tuple[list[int], list[int]]:
    """Disjoint host cores for the CPU expert workers of each rank on one node: the allowed
    cores are split evenly over the node's ranks; each rank keeps its slice's first core for
    its launching thread (one rank alone keeps two) and gives the rest to its workers.
    Returns (worker cores, launcher cores)."""
    if allowed is None:
        allowed = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else []
    if local_world <= 1:
        return (allowed[2:] if len(allowed) > 4 else allowed), allowed[:2]
    n = len(allowed)
    part = allowed[local_rank * n // local_world: (local_rank + 1) * n // local_world]
    if len(part) < 2:
        return part, part
    return part[1:], part[:1]


def balanced_share(threads: int, local_world: int, mode: int | None = None) -> float:
    """CPU share of the host tier that makes the CPU workers and the PCIe reads of one rank
    finish together (the two run at the same time during a layer); `mode` is the CPU kernel
    family (default: the one the pool will use)."""
    if mode is None:
        mode = ext().cpu_gemv_mode()
    cpu = threads * CPU_GBS_PER_THREAD.get(mode, 0.5)
    if local_world > 1:
        cpu = min(cpu, CPU_GBS_PER_RANK_SHARED)
    pcie = PCIE_GBS_ALONE if local_world <= 1 else PCIE_GBS_SHARED if local_world <= 4 else PCIE_GBS_PAIRED
    return round(cpu / (cpu + pcie), 2)


class CpuExpertTier:
    """Owns the mailbox, the CPU thread pool and the split of each layer's host experts."""

    def __init__(self, cache, cfg, max_rows: int, cpu_share: float = 0.75, threads: int | None = None,
                 cpus: list[int] | None = None, timeout_s: float = 2.0, mode: int = -1, ep=None):
        self.cache, self.cfg = cache, cfg
        self.ep = ep  # parallel.ep.EPGroup: this rank's experts for the rows every rank dispatched
        self.E, self.k, self.H, self.I = cfg.n_experts, cfg.top_k, cfg.hidden, cfg.moe_ffn
        if ep is not None:  # the mailbox carries the owner's CSR over its local experts
            self.E = ep.E_loc
            max_rows = ep.N * ep.cap
        self.max_rows = max_rows
        self.cpu_share = cpu_share
        self.timeout_s = timeout_s
        self.device = cache.device
        lay = ext().cpu_mailbox_bytes(self.E, self.k, max_rows, self.H)
        self.mailbox = torch.zeros(lay[-1], dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        self.mb_ptr = self.mailbox.data_ptr()
        self.ctr = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        if cpus is None:
            allowed = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else []
            # the launching thread and the driver keep the first cores
            cpus = allowed[2:] if len(allowed) > 4 else allowed
        if threads is None:
            threads = int(os.environ.get("SYN_CPU_EXPERT_THREADS", max(1, len(cpus))))
        self.threads = threads
        self.native = ext().CpuExpertTier(len(cache.layers), self.E, self.H, self.I, self.k, max_rows,
                                          self.mb_ptr, list(cpus), threads, mode)
        self.layer_of = {id(L): li for li, L in enumerate(cache.layers)}
        cache.cpu_tier = self
        self.assign()
        self.native.start()

    # ------------------------------------------------------------------ split
    def assign(self):
        """Give the CPU `cpu_share` of every layer's host experts (by index order, after the
        cache's residency decisions); the GPU's pointer tables get nulls for them."""
        for li, b in enumerate(self.cache.banks):
            # the CPU takes the host experts with the lowest host rows, so the rows the GPU
            # reads stay one contiguous range (bulk DMA staging copies them in one piece)
            host = sorted((e for e in range(b.E) if b.slot_of[e] < 0), key=lambda e: b.host_of[e])
            n_cpu = int(round(self.cpu_share * len(host)))
            mine = set(host[:n_cpu])
            b.cpu_owned = mine
            for e in range(b.E):
                eg = e if self.ep is not None else b.e0 + e  # local ids under expert parallelism
                if e in mine:
                    h = b.host_of[e]
                    gu, dn = b.parts
                    self.native.set_expert(li, eg, gu["qh"][h].data_ptr(), gu["sh"][h].data_ptr(),
                                           dn["qh"][h].data_ptr(), dn["sh"][h].data_ptr())
                else:
                    self.native.set_expert(li, eg, 0, 0, 0, 0)
            b.rewrite_ptrs()

    def owns_layer(self, L) -> bool:
        li = self.layer_of.get(id(L))
        return li is not None and bool(self.cache.banks[li].cpu_owned)

    # ------------------------------------------------------------------ per layer (decode)
    def handoff(self, L, h, mb):
        """Publish layer L's rows (bf16 [B, H]) and routing CSR to the CPU threads."""
        ext().cpu_handoff(h, mb["tok_off"], mb["tok_idx"], mb["pair_w"], self.E, self.k, self.max_rows,
                          self.mb_ptr, self.layer_of[id(L)], self.ctr)

    def handoff_ep(self, layer_of_cache: int, recv_x, tok_off, tok_idx, pair_w):
        """Expert parallelism: publish every rank's rows received for this rank's experts
        (bf16 [N * cap, H]) and the owner CSR built by ep_build."""
        ext().cpu_handoff(recv_x, tok_off, tok_idx, pair_w, self.E, self.k, self.max_rows, self.mb_ptr,
                          layer_of_cache, self.ctr)

    def collect_ep(self, pair_dst, layer: int):
        """Expert parallelism: wait for the CPU's rows, store each into its source rank's
        combine slot (pair_dst, over NVLink), then raise this layer's completion flags on every
        rank (the down-projection GEMV of this layer left them to this kernel)."""
        ep = self.ep
        ext().cpu_collect_ep(self.mb_ptr, self.E, self.k, self.max_rows, self.H, self.ctr, pair_dst,
                             self.timeout_s, self.status, ep.region.peers, ep.off_flag_comb, ep.rank, ep.step_ctr,
                             ep.n_layers, layer, ep.collect_ctr)

    def collect(self, yp):
        """Wait for the CPU's rows and place them into the pair outputs yp (f32 [B*k, H])."""
        ext().cpu_collect(self.mb_ptr, self.E, self.k, self.max_rows, self.ctr, yp, self.timeout_s, self.status)

    def check(self):
        """Raise if a hand-off timed out or the CPU rejected its input (device status word)."""
        s = int(self.status.item())
        if s:
            from ..core.errors import KERNELS_DOORBELL_TIMEOUT, Domain, ErrorClass, SynError
            self.status.zero_()
            raise SynError(ErrorClass.TIMEOUT, f"CPU expert tier: status {s:#x} (1: no answer within "
                           f"{self.timeout_s} s, 2: the CPU rejected the hand-off)", Domain.KERNELS,
                           KERNELS_DOORBELL_TIMEOUT)

    def stats(self) -> dict:
        return dict(self.native.stats())

    def detach(self):
        """Hand every expert back to the GPU and stop the threads.  Decode graphs captured with
        the hand-off must be captured again (the caller clears them)."""
        for b in self.cache.banks:
            b.cpu_owned = set()
            b.rewrite_ptrs()
        if self.cache.cpu_tier is self:
            self.cache.cpu_tier = None
        self.native.stop()

    def close(self):
        self.native.stop()
