"""VRAM expert cache over a pinned host tier.

Every MoE layer keeps ``n_resident = floor(frac * E_loc)`` experts in VRAM slots; the
others live in pinned host memory, which under unified addressing the GPU reads directly
over PCIe.  The grouped GEMV takes a per-expert pointer table, so an expert's "home" is
just the pointer it is given: a VRAM slot (hit) or its host copy (miss, read in place
while the resident experts stream from HBM on other SMs).

Residency adapts: routing counts feed a decayed LFU score per expert (``ExpertStats``);
``rebalance`` swaps the coldest resident for the hottest host expert when the hot one
leads by a hysteresis margin, copying weights on a side stream between steps.

Reference design: plan/rfcs/RFC-0023-moe-expert-cache-prediction-prefetch.md §5-§9 and
crates/tier/src/experts/{sizing.rs:98-166,stats.rs:35-205}.
"""
from __future__ import annotations

import math

import torch


class ExpertStats:
    """Decayed-LFU expert popularity per layer (counts of routed rows)."""

    def __init__(self, n_layers: int, n_experts: int, decay: float = 0.98, device="cpu"):
        self.decay = decay
        self.score = torch.zeros(n_layers, n_experts, dtype=torch.float64)
        self.total = torch.zeros(n_layers, n_experts, dtype=torch.int64)

    def observe(self, layer: int, counts: torch.Tensor):
        c = counts.detach().to("cpu", torch.float64)
        self.score[layer].mul_(self.decay).add_(c)
        self.total[layer] += counts.detach().to("cpu", torch.int64)

    def hit_rate(self, layer: int, resident: torch.Tensor) -> float:
        t = self.total[layer].double()
        s = t.sum()
        return float((t * resident.double()).sum() / s) if s > 0 else 0.0

    def state_dict(self):
        return {"score": self.score.clone(), "total": self.total.clone(), "decay": self.decay}

    def load_state_dict(self, d):
        self.score.copy_(d["score"])
        self.total.copy_(d["total"])
        self.decay = float(d["decay"])

    def save(self, path: str, model: str = ""):
        """Persist the popularity profile (next to the model pack), so a restarted instance
        starts with the hot experts resident instead of relearning them."""
        torch.save({"model": model, **self.state_dict()}, path)

    @classmethod
    def load(cls, path: str, model: str = "") -> "ExpertStats":
        d = torch.load(path, map_location="cpu", weights_only=False)
        if model and d.get("model") and d["model"] != model:
            raise ValueError(f"expert profile is for {d['model']}, not {model}")
        st = cls(d["score"].shape[0], d["score"].shape[1], d["decay"])
        st.load_state_dict(d)
        return st


class ExpertCache:
    """Residency manager for the expert banks of a model's MoE layers on one device."""

    def __init__(self, layers, frac: float, device, hysteresis: float = 1.25):
        self.layers = [L for L in layers if getattr(L, "is_moe", False)]
        self.frac = frac
        self.device = device
        self.hysteresis = hysteresis
        self.banks = []
        for L in self.layers:
            b = _TieredBank(L.experts_gu, L.experts_down, frac, device)
            self.banks.append(b)
            L.expert_tier = b
        self._staging = None
        self.prefetch = False
        self.stage_all = False  # decode: DMA-stage every GPU-read host expert of each layer
        self.cpu_tier = None  # experts.cpu_tier.CpuExpertTier when host experts run on the CPU
        # CTAs of the prefetch kernel (the rest of the GPU stays with the current layer)
        self.prefetch_ctas = int(__import__("os").environ.get("SYN_PREFETCH_CTAS", "64"))

    # ------------------------------------------------------------------ staging banks
    def _ensure_staging(self):
        if self._staging is not None:
            return
        b = next(x for x in self.banks if x.E > x.n_res)
        # both staging banks are carved out of one VRAM slab by the native arena
        from .._ext import ext
        sizes = [(p["qh"].nbytes, p["sh"].nbytes) for p in b.parts] * 2
        total = sum(q + s_ + 512 for q, s_ in sizes)
        self._arena = ext().Arena(total)
        self._slab = torch.empty(total, dtype=torch.uint8, device=self.device)

        def carve(like):
            off = self._arena.alloc(like.nbytes, 256)
            assert off >= 0
            return self._slab[off: off + like.nbytes].view(like.dtype).view(like.shape)
        self._staging = [[{"q": carve(p["qh"]), "s": carve(p["sh"])} for p in b.parts] for _ in range(2)]
        self._copy_stream = torch.cuda.Stream(device=self.device)
        self._ev_free = [None, None]
        self._issued = {}
        self._last = None

    # ------------------------------------------------------------------ decode prefetch
    def enable_decode_prefetch(self, n_experts: int):
        """Router-predicted prefetch for decode: after layer i routes, the experts it predicts
        for layer i+1 that live in the host tier are copied into a VRAM staging bank on a side
        stream, and layer i+1's pointer tables are pointed at the copies (csrc/cuda/
        expert_prefetch.cu).  Each bank keeps its home pointer tables to fall back on."""
        if not any(b.E > b.n_res for b in self.banks):
            return False
        self._ensure_staging()
        for b in self.banks:
            b.refresh_home()
            b.pred = torch.zeros(n_experts, dtype=torch.int32, device=self.device)
        self.prefetch = True
        return True

    def enable_decode_staging(self):
        """Bulk staging for decode at large batches (when most experts of a layer are routed to
        anyway): every host expert the GPU reads (those the host CPU does not compute) is copied
        by the DMA engines into a VRAM staging bank, layer by layer, double-buffered across
        layers; the live pointer tables point at the staged rows.  The CPU tier takes the lowest
        host rows, so the copied rows of a layer are one contiguous range (4 copies per layer)
        however residency changes.  Replaces the router-predicted prefetch (whose per-expert
        kernel copies are slower than DMA once nearly every expert is predicted)."""
        if not any(b.E > b.n_res for b in self.banks):
            return False
        self._ensure_staging()
        self.prefetch = False
        self.stage_all = True
        self._stage_events = {}
        for li, b in enumerate(self.banks):
            b.stage = self._staging[li % 2]
            b.rewrite_ptrs()
        return True

    def stage_rows(self, li: int) -> int:
        """First host row of layer li that the GPU reads (rows below it belong to the CPU)."""
        b = self.banks[li]
        return len(b.cpu_owned)

    def issue_stage_copy(self, li: int):
        """Copies layer li's GPU-read host rows into its staging bank on the current stream."""
        b = self.banks[li]
        r0 = self.stage_rows(li)
        nh = b.E - b.n_res
        if r0 >= nh:
            return
        for which, p in enumerate(b.parts):
            if p is None:
                continue
            st = b.stage[which]
            st["q"][r0:nh].copy_(p["qh"][r0:nh], non_blocking=True)
            st["s"][r0:nh].copy_(p["sh"][r0:nh], non_blocking=True)

    def decode_prefetch(self, L):
        """Launch the prefetch of layer L's predicted host experts on the current stream
        (the caller forks a side stream); L.expert_tier.pred must hold the prediction."""
        b = L.expert_tier
        if b.E == b.n_res:
            return
        li = next(i for i, X in enumerate(self.layers) if X is L)
        st = self._staging[li % 2]
        host, stage, live, home = [], [], [], []
        for which, p in enumerate(b.parts):
            host += [p["qh"], p["sh"]]
            stage += [st[which]["q"], st[which]["s"]]
            live += [p["bank"].qw_ptrs, p["bank"].sm_ptrs]
            home += [b.home[which][0], b.home[which][1]]
        from .._ext import ext
        ext().expert_prefetch(b.pred, b.host_row_dev, b.e0, host, stage, live, home, self.prefetch_ctas)

    def promote_all(self):
        """Move every expert to VRAM (cap lifted) without changing the pointer-table
        tensors, so CUDA graphs captured against them stay valid."""
        for L, b in zip(self.layers, self.banks):
            for bank, p in zip((L.experts_gu, L.experts_down), b.parts):
                if p is None:
                    continue
                qf = torch.empty((b.E,) + tuple(p["qv"].shape[1:]), dtype=p["qv"].dtype, device=p["qv"].device)
                sf = torch.empty((b.E,) + tuple(p["sv"].shape[1:]), dtype=p["sv"].dtype, device=p["sv"].device)
                for e in range(b.E):
                    s_ = b.slot_of[e]
                    if s_ >= 0:
                        qf[e].copy_(p["qv"][s_])
                        sf[e].copy_(p["sv"][s_])
                    else:
                        qf[e].copy_(p["qh"][b.host_of[e]], non_blocking=True)
                        sf[e].copy_(p["sh"][b.host_of[e]], non_blocking=True)
                torch.cuda.synchronize()
                bank.qw, bank.sm = qf, sf
                p["qv"], p["sv"] = qf, sf
                qs, ss = qf.stride(0) * 4, sf.stride(0) * 2
                bank.qw_ptrs.copy_(torch.tensor([qf.data_ptr() + e * qs for e in range(b.E)], dtype=torch.int64))
                bank.sm_ptrs.copy_(torch.tensor([sf.data_ptr() + e * ss for e in range(b.E)], dtype=torch.int64))
                bank.bank_contiguous = True
            b.slot_of = list(range(b.E))
            b.host_of = [-1] * b.E
            b.n_res = b.E
        self.frac = 1.0
        self._issued = {}
        self.stage_all = False  # nothing left to stage (captured decode graphs must be captured again)
        for b in self.banks:
            b.stage = None
        for b in self.banks:
            if b.home is not None:  # every expert is home now: the prefetch kernel copies nothing
                b.refresh_home()
        if not self.prefetch:
            self._staging = None
        if self.cpu_tier is not None:  # nothing is left on the host: the CPU owns no expert
            self.cpu_tier.assign()
        torch.cuda.empty_cache()

    def save_host_tier(self, path: str) -> dict:
        """Writes every bank's host-tier rows (tiled 4-bit weights and scales) and the
        residency map as a pack, so a restart reloads the cold experts from disk."""
        from ..store.pack import write_pack
        tensors = {}
        for li, b in enumerate(self.banks):
            for which, p in enumerate(b.parts):
                if p is not None:
                    tensors[f"{li}.{which}.q"] = p["qh"]
                    tensors[f"{li}.{which}.s"] = p["sh"]
        side = write_pack(path, tensors)
        import json
        with open(path + ".residency.json", "w") as f:
            json.dump([{"slot_of": b.slot_of, "host_of": b.host_of} for b in self.banks], f)
        return side

    def load_host_tier(self, path: str, threads: int = 8) -> int:
        """Fills the host tier from a pack written by save_host_tier (direct-I/O reads through the
        native I/O pool).  The residency map must be the one the pack was written with."""
        import json

        from ..store.pack import read_pack_into
        with open(path + ".residency.json") as f:
            res = json.load(f)
        if [(r["slot_of"], r["host_of"]) for r in res] != [(b.slot_of, b.host_of) for b in self.banks]:
            raise ValueError("pack was written with another expert residency")
        targets = {}
        for li, b in enumerate(self.banks):
            for which, p in enumerate(b.parts):
                if p is not None:
                    targets[f"{li}.{which}.q"] = p["qh"]
                    targets[f"{li}.{which}.s"] = p["sh"]
        return read_pack_into(path, targets, threads=threads)

    def staged_ptrs(self, L):
        """Pointer tables with every expert of layer L in VRAM: residents in place, host
        experts copied into one of two staging banks.  Used by prefill, whose GEMM streams
        weights with TMA copies that must read device memory.

        The copies run on a side stream, double-buffered across layers: when layer i asks for
        its tables, the copy of layer i+1's host experts is issued into the other bank, so it
        crosses PCIe while layer i computes.  Layers are asked for in order within one prefill
        pass; a bank is refilled only after the compute stream has passed the layer that read
        it (events)."""
        b = L.expert_tier
        if b.E - b.n_res == 0:
            return (L.experts_gu.qw_ptrs, L.experts_gu.sm_ptrs), (L.experts_down.qw_ptrs, L.experts_down.sm_ptrs)
        if not b.cuda:
            return self._host_ptrs(L)
        self._ensure_staging()
        li = next(i for i, X in enumerate(self.layers) if X is L)
        cur = torch.cuda.current_stream(self.device)
        if self._last is None or li <= self._last:
            # a new prefill pass: the banks may still be read by earlier work (decode-step
            # prefetch copies included), so the copy stream starts after everything enqueued
            self._copy_stream.wait_stream(cur)
        if self._last is not None and self._last in self._issued:
            # every kernel of the previously asked layer is enqueued: its bank is free after them
            ev = torch.cuda.Event()
            ev.record(cur)
            self._ev_free[self._issued[self._last][0]] = ev
        if self._last is not None and li <= self._last:  # a new prefill pass: start over
            self._issued = {}
        self._last = li
        if li not in self._issued:
            self._issue(li, li % 2)
        buf, done = self._issued[li]
        cur.wait_event(done)
        nxt = self.layers[li + 1].expert_tier if li + 1 < len(self.layers) else None
        if nxt is not None and nxt.E > nxt.n_res:
            self._issue(li + 1, 1 - buf)
        self._staged_buf = (li, buf)
        return self._ptrs_for(L, buf)

    def staged_banks(self, L):
        """After `staged_ptrs(L)`: the two contiguous banks that hold layer L's experts for the
        prefill GEMM's tensor maps, per matrix (gate_up, down): (resident q, resident s, staged q,
        staged s), and the selector int32 [E]: (slot << 1) for a resident expert, (host row << 1)
        | 1 for a staged one.  None when the layer is not staged on the device."""
        b = L.expert_tier
        if not b.cuda:
            return None
        li = next(i for i, X in enumerate(self.layers) if X is L)
        if b.E - b.n_res == 0 or getattr(self, "_staged_buf", (None,))[0] != li:
            return None
        buf = self._staged_buf[1]
        sel = [(b.slot_of[e] << 1) if b.slot_of[e] >= 0 else ((b.host_of[e] << 1) | 1) for e in range(b.E)]
        banks = []
        for which, p in enumerate(b.parts):
            st = self._staging[buf][which]
            res_q, res_s = (p["qv"], p["sv"]) if b.n_res > 0 else (st["q"], st["s"])
            banks.append((res_q, res_s, st["q"], st["s"]))
        return banks[0], banks[1], torch.tensor(sel, dtype=torch.int32).to(self.device, non_blocking=True)

    def _issue(self, li, buf):
        b = self.layers[li].expert_tier
        s = self._copy_stream
        if self._ev_free[buf] is not None:
            s.wait_event(self._ev_free[buf])
        with torch.cuda.stream(s):
            for which, p in enumerate(b.parts):
                st = self._staging[buf][which]
                st["q"].copy_(p["qh"], non_blocking=True)
                st["s"].copy_(p["sh"], non_blocking=True)
        done = torch.cuda.Event()
        done.record(s)
        self._issued[li] = (buf, done)

    def _ptrs_for(self, L, buf):
        b = L.expert_tier
        out = []
        for which, p in enumerate(b.parts):
            st = self._staging[buf][which]
            qp, sp = [], []
            for e in range(b.E):
                slot = b.slot_of[e]
                if slot >= 0:
                    qp.append(p["qv"].data_ptr() + slot * p["qv"].stride(0) * 4)
                    sp.append(p["sv"].data_ptr() + slot * p["sv"].stride(0) * 2)
                else:
                    h = b.host_of[e]
                    qp.append(st["q"].data_ptr() + h * st["q"].stride(0) * 4)
                    sp.append(st["s"].data_ptr() + h * st["s"].stride(0) * 2)
            out.append((torch.tensor(qp, dtype=torch.int64, device=self.device),
                        torch.tensor(sp, dtype=torch.int64, device=self.device)))
        return out[0], out[1]

    def _host_ptrs(self, L):
        """CPU banks: the tables point at the resident and host rows themselves."""
        b = L.expert_tier
        out = []
        for p in b.parts:
            qp, sp = [], []
            for e in range(b.E):
                slot = b.slot_of[e]
                src_q, src_s, r = (p["qv"], p["sv"], slot) if slot >= 0 else (p["qh"], p["sh"], b.host_of[e])
                qp.append(src_q.data_ptr() + r * src_q.stride(0) * 4)
                sp.append(src_s.data_ptr() + r * src_s.stride(0) * 2)
            out.append((torch.tensor(qp, dtype=torch.int64), torch.tensor(sp, dtype=torch.int64)))
        return out[0], out[1]

    @property
    def n_resident(self) -> int:
        return self.banks[0].n_res if self.banks else 0

    def vram_bytes(self) -> int:
        return sum(b.vram_bytes() for b in self.banks)

    def host_bytes(self) -> int:
        return sum(b.host_bytes() for b in self.banks)

    def rebalance(self, stats: ExpertStats, max_swaps_per_layer: int = 2) -> int:
        """Swap cold residents for hot host experts (decayed LFU with hysteresis); the plan
        comes from the native planner (`tier_plan_swaps`)."""
        from .._ext import ext
        n = 0
        for li, b in enumerate(self.banks):
            sc = stats.score[li, b.e0: b.e0 + b.E].tolist()
            plan = ext().tier_plan_swaps(sc, b.resident_mask().tolist(), max_swaps_per_layer, self.hysteresis)
            for cold_res, hot_host in plan:
                b.swap(cold_res, hot_host)
                n += 1
        if n and getattr(self, "cpu_tier", None) is not None:
            self.cpu_tier.assign()  # the host set changed: re-split it between the CPU and PCIe
        return n


class _TieredBank:
    """Moves an ExpertBank pair (gate_up, down) to a resident/host split in place."""

    def __init__(self, gu, dn, frac, device):
        self.gu, self.dn = gu, dn
        self.E = gu.E
        self.e0 = gu.e0
        self.home = None
        self.host_row_dev = None
        self.stage = None  # decode bulk staging: [{"q", "s"} per part] this layer's GPU-read host rows live in
        self.cpu_owned: set[int] = set()  # local experts computed by the host CPU (null pointers here)
        self.n_res = max(0, min(self.E, int(math.floor(frac * self.E + 1e-9))))
        self.slot_of = list(range(self.n_res)) + [-1] * (self.E - self.n_res)  # expert -> vram slot
        self.host_of = [-1] * self.n_res + list(range(self.E - self.n_res))    # expert -> host row
        cuda = device.type == "cuda" if hasattr(device, "type") else str(device).startswith("cuda")
        self.cuda = cuda
        self.parts = []
        for bank in (gu, dn):
            if bank.qw is None:
                self.parts.append(None)
                continue
            nh = self.E - self.n_res
            qh = torch.empty((nh,) + tuple(bank.qw.shape[1:]), dtype=bank.qw.dtype, pin_memory=cuda)
            sh = torch.empty((nh,) + tuple(bank.sm.shape[1:]), dtype=bank.sm.dtype, pin_memory=cuda)
            if nh:
                qh.copy_(bank.qw[self.n_res:])
                sh.copy_(bank.sm[self.n_res:])
            qv = bank.qw[: self.n_res].clone()
            sv = bank.sm[: self.n_res].clone()
            bank.qw, bank.sm = qv, sv  # VRAM keeps only the resident slots
            bank.bank_contiguous = False
            self.parts.append({"bank": bank, "qv": qv, "sv": sv, "qh": qh, "sh": sh})
            self._write_ptrs(bank, qv, sv, qh, sh)
        if cuda:
            torch.cuda.empty_cache()

    def _write_ptrs(self, bank, qv, sv, qh, sh, stage=None):
        qp, sp = [], []
        for e in range(self.E):
            s = self.slot_of[e]
            if e in self.cpu_owned:  # the GEMVs skip experts with a null weight pointer
                qp.append(0)
                sp.append(0)
            elif s >= 0:
                qp.append(qv.data_ptr() + s * qv.stride(0) * qv.element_size())
                sp.append(sv.data_ptr() + s * sv.stride(0) * sv.element_size())
            else:
                h = self.host_of[e]
                tq, ts = (stage["q"], stage["s"]) if stage is not None else (qh, sh)
                qp.append(tq.data_ptr() + h * tq.stride(0) * tq.element_size())
                sp.append(ts.data_ptr() + h * ts.stride(0) * ts.element_size())
        dev = bank.qw_ptrs.device if bank.qw_ptrs is not None else qv.device
        new_q = torch.tensor(qp, dtype=torch.int64)
        new_s = torch.tensor(sp, dtype=torch.int64)
        if bank.qw_ptrs is None:
            bank.qw_ptrs, bank.sm_ptrs = new_q.to(dev), new_s.to(dev)
        else:  # in place: captured graphs keep reading the same pointer tables
            bank.qw_ptrs.copy_(new_q)
            bank.sm_ptrs.copy_(new_s)

    def _stage_of(self, which):
        return self.stage[which] if self.stage is not None else None

    def rewrite_ptrs(self):
        """Rewrite the live pointer tables in place (after a change of ownership)."""
        for which, p in enumerate(self.parts):
            if p is not None:
                self._write_ptrs(p["bank"], p["qv"], p["sv"], p["qh"], p["sh"], self._stage_of(which))
        if self.home is not None:
            self.refresh_home()

    def refresh_home(self):
        """Snapshot the home pointer tables (resident slot or host row per expert) and the
        host-row map used by the decode prefetch kernel."""
        # experts the host CPU computes are never staged (the GPU skips them)
        rows = torch.tensor([self.host_of[e] if self.slot_of[e] < 0 and e not in self.cpu_owned else -1
                             for e in range(self.E)], dtype=torch.int32)
        if self.home is None:
            self.home = [(p["bank"].qw_ptrs.clone(), p["bank"].sm_ptrs.clone()) if p is not None else None
                         for p in self.parts]
            self.host_row_dev = rows.to(self.parts[0]["bank"].qw_ptrs.device)
        else:  # in place: captured decode graphs keep reading these tensors
            for p, hm in zip(self.parts, self.home):
                if p is not None:
                    hm[0].copy_(p["bank"].qw_ptrs)
                    hm[1].copy_(p["bank"].sm_ptrs)
            self.host_row_dev.copy_(rows)

    def resident_mask(self) -> torch.Tensor:
        return torch.tensor([s >= 0 for s in self.slot_of])

    def vram_bytes(self):
        return sum(p["qv"].numel() * 4 + p["sv"].numel() * 2 for p in self.parts if p)

    def host_bytes(self):
        return sum(p["qh"].numel() * 4 + p["sh"].numel() * 2 for p in self.parts if p)

    def swap(self, e_res: int, e_host: int):
        """Exchange the homes of a resident and a host expert (weights copied both ways)."""
        s, h = self.slot_of[e_res], self.host_of[e_host]
        for p in self.parts:
            if p is None:
                continue
            tq = p["qv"][s].clone()
            ts = p["sv"][s].clone()
            p["qv"][s].copy_(p["qh"][h], non_blocking=True)
            p["sv"][s].copy_(p["sh"][h], non_blocking=True)
            p["qh"][h].copy_(tq, non_blocking=False)
            p["sh"][h].copy_(ts, non_blocking=False)
        self.slot_of[e_res], self.slot_of[e_host] = -1, s
        self.host_of[e_res], self.host_of[e_host] = h, -1
        for which, p in enumerate(self.parts):
            if p is not None:
                self._write_ptrs(p["bank"], p["qv"], p["sv"], p["qh"], p["sh"], self._stage_of(which))
        if self.home is not None:
            self.refresh_home()

    def weight_of(self, which: int, e: int):
        """Dense view of expert e (for the CPU path / tests)."""
        p = self.parts[which]
        s = self.slot_of[e]
        return (p["qv"][s], p["sv"][s]) if s >= 0 else (p["qh"][self.host_of[e]], p["sh"][self.host_of[e]])
