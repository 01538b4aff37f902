"""CPU oracle of the device sampler (csrc/cuda/sampler.cu): same Philox4x32-10 draw
contract, same fixed-point inverse-CDF selection, same top-k/top-p thresholds."""
from __future__ import annotations

import math

import torch

M0, M1 = 0xD2511F53, 0xCD9E8D57
W0, W1 = 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32_10(ctr: list[int], k0: int, k1: int) -> list[int]:
    """Philox4x32-10 from Salmon et al., SC'11 (pure Python)."""
    c = list(ctr)
    for r in range(10):
        if r:
            k0 = (k0 + W0) & MASK
            k1 = (k1 + W1) & MASK
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        hi0, lo0 = p0 >> 32, p0 & MASK
        hi1, lo1 = p1 >> 32, p1 & MASK
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
    return c


def philox_draw(seed: int, stream: int, counter: int) -> int:
    seed &= (1 << 64) - 1
    stream &= (1 << 64) - 1
    counter &= (1 << 64) - 1
    c = philox4x32_10([counter & MASK, counter >> 32, stream & MASK, stream >> 32], seed & MASK, seed >> 32)
    return c[0]


def sample_row(logits: torch.Tensor, temperature: float, top_k: int, top_p: float, seed: int, stream: int,
               counter: int) -> tuple[int, int]:
    """Returns (token, new_counter)."""
    lg = logits.double() if False else logits.float()
    if not temperature > 0:
        return int(torch.argmax(lg).item()), counter
    z = lg / temperature
    mx = z.max()
    V = z.numel()
    keep = torch.ones(V, dtype=torch.bool)
    if 0 < top_k < V:
        kth = torch.sort(z, descending=True).values[top_k - 1]
        keep &= z >= kth
    mass = torch.where(keep, torch.floor(torch.exp(z - mx).double() * 4294967296.0), torch.zeros(V, dtype=torch.float64))
    mass = mass.to(torch.int64)
    if top_p < 1.0:
        total = int(mass.sum())
        need = int(top_p * total)
        vals = torch.sort(mass, descending=True).values
        cum = torch.cumsum(vals, 0)
        idx = int(torch.searchsorted(cum, torch.tensor(need)).item())
        idx = min(idx, V - 1)
        floor = int(vals[idx])
        mass = torch.where(mass >= floor, mass, torch.zeros_like(mass))
    total = int(mass.sum())
    x0 = philox_draw(seed, stream, counter)
    target = (x0 * total) >> 32
    cum = torch.cumsum(mass, 0)
    tok = int(torch.searchsorted(cum, torch.tensor(target), right=True).item())
    return min(tok, V - 1), counter + 1


def sample_ref(logits, temperature, top_k, top_p, seed, stream, counter) -> torch.Tensor:
    T = logits.shape[0]
    out = torch.empty(T, dtype=torch.int32)
    for t in range(T):
        tok, c = sample_row(logits[t], float(temperature[t]), int(top_k[t]), float(top_p[t]), int(seed[t]),
                            int(stream[t]), int(counter[t]))
        out[t] = tok
        counter[t] = c
    return out


def _row_masses(lg: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    z = lg.float() / temperature
    V = z.numel()
    keep = torch.ones(V, dtype=torch.bool)
    if 0 < top_k < V:
        keep &= z >= torch.sort(z, descending=True).values[top_k - 1]
    mass = torch.where(keep, torch.floor(torch.exp(z - z.max()).double() * 4294967296.0),
                       torch.zeros(V, dtype=torch.float64)).to(torch.int64)
    if top_p < 1.0:
        total = int(mass.sum())
        need = int(top_p * total)
        vals = torch.sort(mass, descending=True).values
        idx = min(int(torch.searchsorted(torch.cumsum(vals, 0), torch.tensor(need)).item()), V - 1)
        mass = torch.where(mass >= int(vals[idx]), mass, torch.zeros_like(mass))
    return mass


def _draw(mass: torch.Tensor, x0: int) -> int:
    total = int(mass.sum())
    target = (x0 * total) >> 32
    tok = int(torch.searchsorted(torch.cumsum(mass, 0), torch.tensor(target), right=True).item())
    return min(tok, mass.numel() - 1)


_U64 = (1 << 64) - 1


def _norm32(masses: list[int]) -> list[int]:
    """Fixed-point masses -> probabilities in units of 2^-32 (the device's exact integer rule:
    r = floor((2^64 - 1) / total), each (m * r) >> 32)."""
    tot = sum(masses)
    if tot == 0:
        return [0] * len(masses)
    r = _U64 // tot
    return [(m * r) >> 32 for m in masses]


def _draft_masses(q: torch.Tensor) -> list[int]:
    """Draft probabilities (f32) -> fixed-point masses floor(q * 2^32) (negative / NaN -> 0)."""
    qd = q.float().double()
    return [int(math.floor(v * 4294967296.0)) if v > 0 else 0 for v in qd.tolist()]


def _draw_list(mass: list[int], x0: int) -> int:
    total = sum(mass)
    target = (x0 * total) >> 32
    run = 0
    for i, m in enumerate(mass):
        if m and run + m > target:
            return i
        run += m
    return 0


def verify_ref(logits, draft, temperature, top_k, top_p, seed, stream, counter, draft_probs=None):
    """Host oracle of the device VerifyAccept kernel.
    logits [S*(g+1), V], draft [S, g] -> (tokens [S, g+1], n_accept [S]); counter updated.
    draft_probs None: point-mass drafts (accept iff u < p(d); residual p without d).
    draft_probs [S, g, V]: drafts sampled from those distributions q (accept iff
    u < min(1, p(d) / q(d)); residual norm(max(0, p - q))), in the device's exact integers."""
    S, g = draft.shape
    out = torch.zeros(S, g + 1, dtype=torch.int32)
    nacc = torch.zeros(S, dtype=torch.int32)
    for s in range(S):
        t = float(temperature[s])
        ctr = int(counter[s])
        n = g
        for j in range(g + 1):
            lg = logits[s * (g + 1) + j]
            dj = int(draft[s, j]) if j < g else -1
            if not t > 0:
                a = int(torch.argmax(lg).item())
                if j < g and a == dj:
                    out[s, j] = dj
                    continue
                out[s, j] = a
                n = min(j, g)
                break
            mass = _row_masses(lg, t, int(top_k[s]), float(top_p[s]))
            if j < g and draft_probs is not None:
                u = philox_draw(int(seed[s]), int(stream[s]), ctr)
                ctr += 1
                pn = _norm32(mass.tolist())
                qn = _norm32(_draft_masses(draft_probs[s, j]))
                if 0 <= dj < len(pn) and u * qn[dj] < (pn[dj] << 32):
                    out[s, j] = dj
                    continue
                res = [a - b if a > b else 0 for a, b in zip(pn, qn)]
                if not any(res):  # p == q up to rounding: the residual is p itself
                    res = pn
                out[s, j] = _draw_list(res, philox_draw(int(seed[s]), int(stream[s]), ctr))
                ctr += 1
                n = j
                break
            if j < g:
                u = philox_draw(int(seed[s]), int(stream[s]), ctr)
                ctr += 1
                if (u * int(mass.sum())) >> 32 < int(mass[dj]):
                    out[s, j] = dj
                    continue
                m2 = mass.clone()
                m2[dj] = 0
                out[s, j] = _draw(m2, philox_draw(int(seed[s]), int(stream[s]), ctr))
                ctr += 1
                n = j
                break
            out[s, j] = _draw(mass, philox_draw(int(seed[s]), int(stream[s]), ctr))
            ctr += 1
            n = g
        nacc[s] = n
        counter[s] = ctr
    return out, nacc
