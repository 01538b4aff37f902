"""Device-dispatched ops (CUDA kernel or CPU f32 torch)."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .._ext import ext
from ..formats.q4 import Q4Weight

__all__ = [
    "GEMV_STORE", "GEMV_SWIGLU", "GEMV_SCALED_F32", "GEMV_ADD_F32",
    "rms_norm", "embed", "linear", "linear_grouped", "qk_rope_kv_write", "attn_decode",
    "attn_prefill", "attn_prefill_paged", "mla_decode", "router_logits", "doorbell_wait", "doorbell_ring",
    "timestamp", "tap_rows", "tap_compare", "kv_pack", "kv_unpack", "moe_topk", "moe_combine_rmsnorm", "argmax", "sample",
    "swiglu_interleaved_ref", "interleave_gate_up", "count_launches", "DECODE_ROWS_MAX", "moe_nt_hint", "gemm_grouped", "gemm_status", "block_sums",
]

GEMV_STORE, GEMV_SWIGLU, GEMV_SCALED_F32, GEMV_ADD_F32 = 0, 1, 2, 3
DECODE_ROWS_MAX = 64  # above this a linear runs as a GEMM


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[f, K] x2 -> [2f, K] with 8-row gate/up chunks: rows 16c..16c+7 = gate[8c..8c+7],
    rows 16c+8..16c+15 = up[8c..8c+7] (the layout the SWIGLU GEMV epilogue reads)."""
    f, K = gate.shape
    assert f % 8 == 0
    return torch.stack([gate.reshape(f // 8, 8, K), up.reshape(f // 8, 8, K)], dim=1).reshape(2 * f, K)


def swiglu_interleaved_ref(gu: torch.Tensor) -> torch.Tensor:
    T, n2 = gu.shape
    g = gu.reshape(T, n2 // 16, 2, 8)
    return (F.silu(g[:, :, 0].float()) * g[:, :, 1].float()).reshape(T, n2 // 2)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    if x.is_cuda:
        if out is None:
            out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        ext().rmsnorm(x, w, eps, out)
        _launched()
        return out
    x32 = x.float()
    y = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    if out is not None:
        out.copy_(y)
        return out
    return y


def embed(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    if table.is_cuda:
        ext().embed(table, ids, out)
        _launched()
    else:
        out.copy_(table.float()[ids.long()])
    return out


_LAUNCHES = {"count": None}


def count_launches(fn) -> int:
    """Runs ``fn`` eagerly and returns how many of this package's kernels it launched."""
    _LAUNCHES["count"] = 0
    try:
        fn()
    finally:
        n = _LAUNCHES["count"]
        _LAUNCHES["count"] = None
    return n


def _launched(n: int = 1):
    if _LAUNCHES["count"] is not None:
        _LAUNCHES["count"] += n


def _dense_weight(W) -> torch.Tensor:
    from ..formats.fp8 import FP8Weight
    return W.dequant() if isinstance(W, (Q4Weight, FP8Weight)) else W


def _f8_ptrs(W):
    p = getattr(W, "_ptrs", None)
    if p is None:
        dev = W.tiled.device
        p = (torch.tensor([W.tiled.data_ptr()], dtype=torch.int64, device=dev),
             torch.tensor([W.scale.data_ptr()], dtype=torch.int64, device=dev))
        W._ptrs = p
    return p


_F8_WS: dict = {}


def _f8_workspace(dev, floats: int) -> torch.Tensor:
    key = str(dev)
    ws = _F8_WS.get(key)
    if ws is None or ws.numel() < floats:
        ws = torch.empty(floats, dtype=torch.float32, device=dev)
        _F8_WS[key] = ws
    return ws


def _linear_fp8(x, W, out, mode):
    """Block-scaled fp8 GEMV: x quantised to e4m3 with 1x128 scales, e4m3 x e4m3 tensor-core
    products, both scales applied per 128-column block."""
    T = x.shape[0]
    kmode = {GEMV_STORE: 0, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
    if kmode == 0 and out.dtype == torch.float32:
        kmode = 5
    xq, xs = ext().f8_quant_act(x if x.stride(-1) == 1 else x.contiguous())
    qp, sp = _f8_ptrs(W)
    # split-K workspace only where the row tiles alone underfill the GPU (< ~4 CTAs per SM)
    ws = _f8_workspace(x.device, 16 * T * W.N) if W.N < 16 * 4 * 148 * 2 else _EMPTY_F32(x.device)
    ext().f8_gemv(xq, xs, qp, sp, _identity_off(T, x.device), _EMPTY_I32(x.device), _EMPTY_F32(x.device), out,
                  W.N, W.K, kmode, (T + 7) // 8, ws)
    _launched(2)
    return out


# SYN_Q4_TC_MIN: fewest token rows for which 4-bit decode products run on tcgen05 (default 32,
# measured: at 16 rows the mma.sync GEMV is still faster, from 32 rows the tcgen05 GEMM; a value
# above 64 keeps every decode product on the GEMV)
_Q4_TC = [int(__import__("os").environ.get("SYN_Q4_TC_MIN", "32"))]


def linear(x: torch.Tensor, W, out: torch.Tensor, mode: int = GEMV_STORE, res: torch.Tensor | None = None):
    """out = x @ W^T with an epilogue:
    STORE: out = y; SWIGLU: out = silu(gate) * up (interleaved rows); ADD_F32: out += y (f32)."""
    if not x.is_cuda:
        y = x.float() @ W.float().t()
        if mode == GEMV_SWIGLU:
            out.copy_(swiglu_interleaved_ref(y))
        elif mode == GEMV_ADD_F32:
            out.add_(y)
        else:
            out.copy_(y)
        return out
    T = x.shape[0]
    if getattr(W, "tiled", None) is not None and T <= DECODE_ROWS_MAX and x.dtype == torch.bfloat16:
        return _linear_fp8(x, W, out, mode)
    if isinstance(W, Q4Weight) and _Q4_TC[0] <= T <= DECODE_ROWS_MAX and W.N % 128 == 0 and W.K % 64 == 0 and \
            x.dtype == torch.bfloat16 and x.stride(-1) == 1 and out.stride(-1) == 1:
        # 16-64 rows: tcgen05 with the dequantised weights as the M operand (one dequantisation
        # per weight whatever the row count; the mma.sync GEMV is instruction-bound here)
        kmode = {GEMV_STORE: 0 if out.dtype == torch.bfloat16 else 5, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
        ext().q4_gemm_dec(x, W.qw, W.sm, W.N, W.K, kmode, out, gemm_status(x.device))
        _launched()
        return out
    if isinstance(W, Q4Weight) and (_DENSE_V5[1] <= T or W.N * W.K >= (64 << 20)) and T <= DECODE_ROWS_MAX \
            and W.N % 64 == 0 and W.K % 128 == 0 and _DENSE_V5[0]:
        kmode = {GEMV_STORE: 0, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
        if kmode == 0 and out.dtype == torch.float32:
            kmode = 5
        ws, ctr = _dense_workspace(x.device, W.N, T, W.K)
        ptrs = _ptrs(W)
        ext().q4_gemv_dense(x, ptrs[0], ptrs[1], _identity_off(T, x.device), out, W.N, W.K, kmode, ws, ctr)
        _launched()
        return out
    if isinstance(W, Q4Weight) and T <= DECODE_ROWS_MAX and T > 8 and _DENSE_AS_GROUPS[0]:
        # token groups of 8 over shared weights: one HBM pass, the other groups hit L2
        kmode = {GEMV_STORE: 0, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
        if kmode == 0 and out.dtype == torch.float32:
            kmode = 5
        qp, sp, off = _group_ptrs(W, T)
        ext().q4_gemv(x, qp, sp, off, _EMPTY_I32(x.device), _EMPTY_F32(x.device), _EMPTY_BF16(x.device), out, W.N,
                      W.K, kmode, 1, qp.numel(), _EMPTY_F32(x.device), True)
        _launched()
        return out
    if isinstance(W, Q4Weight) and T <= DECODE_ROWS_MAX:
        ptrs = _ptrs(W)
        kmode = {GEMV_STORE: 0, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
        if kmode == 0 and out.dtype == torch.float32:
            kmode = 5
        ext().q4_gemv(x, ptrs[0], ptrs[1], _identity_off(T, x.device), _EMPTY_I32(x.device), _EMPTY_F32(x.device),
                      _EMPTY_BF16(x.device), out, W.N, W.K, kmode, (T + 7) // 8, 1, _EMPTY_F32(x.device), True)
        _launched()
        return out
    # GEMM path (prefill): tcgen05 kernel with fused dequant and epilogue
    if isinstance(W, Q4Weight) and W.N % 128 == 0 and W.K % 64 == 0:
        ptrs = _ptrs(W)
        gm = {GEMV_STORE: 0 if out.dtype == torch.bfloat16 else 5, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
        gemm_grouped(x, ptrs[0], ptrs[1], _identity_off(T, x.device), W.N, W.K, gm, None, out, 1, W.qw, W.sm)
        return out
    if isinstance(W, torch.Tensor) and W.dtype == torch.bfloat16 and x.dtype == torch.bfloat16 and \
            W.shape[0] % 32 == 0 and W.shape[1] % 64 == 0 and x.stride(-1) == 1 and \
            (mode != GEMV_SWIGLU or W.shape[0] % 16 == 0) and _bf16_provider(x, W, mode) == "tcgen05":
        # bf16 weights: tcgen05 GEMM (decode orientation with split-K below 128 rows)
        N, K = W.shape
        gm = {GEMV_STORE: 0 if out.dtype == torch.bfloat16 else 5, GEMV_SWIGLU: 1, GEMV_ADD_F32: 3}[mode]
        ws, ctr = _bf16_workspace(x.device, N, K, T)
        ext().gemm_bf16(x, W if W.is_contiguous() else W.contiguous(), out, gm, ws, ctr, gemm_status(x.device))
        _launched()
        return out
    if getattr(W, "tiled", None) is not None and x.dtype == torch.bfloat16 and W.N % 32 == 0 and \
            (mode != GEMV_SWIGLU or W.N % 16 == 0):
        # prefill over block-scaled fp8 weights: widened to bf16 (scales applied) in one pass,
        # then the tcgen05 GEMM
        return linear(x, ext().f8_dequant_tiled(W.tiled, W.scale, W.N, W.K), out, mode)
    Wd = _dense_weight(W)
    y = x.to(Wd.dtype) @ Wd.t()
    if mode == GEMV_SWIGLU:
        out.copy_(swiglu_interleaved_ref(y))
    elif mode == GEMV_ADD_F32:
        out.add_(y.float())
    else:
        out.copy_(y)
    return out


# bf16 GEMM provider: "1" the tcgen05 kernel, "0" the library GEMM, "auto" chosen per shape by
# the selector (certified against the f32 reference, then timed; 3% margin for the default)
_BF16_TC = [__import__("os").environ.get("SYN_BF16_TC", "1")]
SELECTOR = None


def _bf16_provider(x, W, mode) -> str:
    choice = _BF16_TC[0]
    if choice != "auto":
        return "tcgen05" if choice == "1" else "library"
    global SELECTOR
    from .numerics import Candidate, Selector
    if SELECTOR is None:
        SELECTOR = Selector()
    T = x.shape[0]
    bucket = 1 << max(0, (T - 1).bit_length())
    key = f"linear_bf16:{W.shape[0]}x{W.shape[1]}x{bucket}x{mode}"
    if key in SELECTOR.decisions:
        return SELECTOR.decisions[key]
    if torch.cuda.is_current_stream_capturing():
        return "tcgen05"  # decisions are made outside capture (the warm-up passes come first)
    N, K = W.shape
    xs = x.contiguous()

    def ours(a, w):
        o = torch.empty(a.shape[0], N, dtype=torch.float32, device=a.device)
        ws, ctr = _bf16_workspace(a.device, N, K, a.shape[0])
        ext().gemm_bf16(a, w, o, 5, ws, ctr, gemm_status(a.device))
        return o

    def lib(a, w):
        return (a @ w.t()).float()
    pick = SELECTOR.choose("linear_bf16", (N, K, bucket, mode),
                           [Candidate("tcgen05", ours, "bf16_f32acc"), Candidate("library", lib, "bf16_out")],
                           (xs, W if W.is_contiguous() else W.contiguous()),
                           lambda a, w: a.float() @ w.float().t())
    SELECTOR.decisions[key] = pick
    return pick
_BF16_WS: dict = {}


def _bf16_workspace(dev, N: int, K: int, T: int):
    """Split-K workspace (f32) and per-row-tile counters of the bf16 tcgen05 GEMM, grown on
    demand to the largest plan so far on this device (allocated outside graph capture by the
    warm-up passes that precede it)."""
    key = str(dev)
    need = max(0, ext().gemm_bf16_ws(N, K, T))
    ws, ctr = _BF16_WS.get(key, (None, None))
    tiles = (N + 127) // 128
    if ws is None or ws.numel() < need or ctr.numel() < tiles:
        ws = torch.empty(max(need, ws.numel() if ws is not None else 0), dtype=torch.float32, device=dev)
        ctr = torch.zeros(max(tiles, ctr.numel() if ctr is not None else 0), dtype=torch.int32, device=dev)
        _BF16_WS[key] = (ws, ctr)
    return ws, ctr


_PTR_CACHE: dict = {}
_GROUP_CACHE: dict = {}
# dense decode GEMV: split-K smem-staged kernel (v5) for rows in [SYN_DENSE_V5_MIN, 64]
_DENSE_V5 = [__import__("os").environ.get("SYN_DENSE_V5", "1") == "1",
             int(__import__("os").environ.get("SYN_DENSE_V5_MIN", "9"))]
_DENSE_WS: dict = {}


def _dense_workspace(dev, N: int, T: int, K: int):
    """Split-K workspace (f32) and arrival counters of the dense GEMV, grown on demand to the
    largest split planned so far on this device."""
    key = str(dev)
    need = max(0, ext().q4_gemv_dense_ws(N, K, min(T, 64)))
    ws, ctr = _DENSE_WS.get(key, (None, None))
    if ws is None or ws.numel() < need or ctr.numel() < N // 64:
        ws = torch.empty(max(need, ws.numel() if ws is not None else 1), dtype=torch.float32, device=dev)
        ctr = torch.zeros(max(N // 64, ctr.numel() if ctr is not None else 0), dtype=torch.int32, device=dev)
        _DENSE_WS[key] = (ws, ctr)
    return ws, ctr
_DENSE_AS_GROUPS = [__import__("os").environ.get("SYN_DENSE_GROUPS", "0") == "1"]


def _group_ptrs(W: Q4Weight, T: int):
    key = (W.qw.data_ptr(), T)
    v = _GROUP_CACHE.get(key)
    if v is None:
        G = (T + 7) // 8
        dev = W.qw.device
        v = (torch.tensor([W.qw.data_ptr()] * G, dtype=torch.int64, device=dev),
             torch.tensor([W.sm.data_ptr()] * G, dtype=torch.int64, device=dev),
             torch.tensor([min(8 * g, T) for g in range(G + 1)], dtype=torch.int32, device=dev))
        _GROUP_CACHE[key] = v
    return v
_OFF_CACHE: dict = {}
_EMPTY: dict = {}


def _ptrs(W: Q4Weight):
    key = (W.qw.data_ptr(), W.sm.data_ptr())
    p = _PTR_CACHE.get(key)
    if p is None:
        dev = W.qw.device
        p = (torch.tensor([W.qw.data_ptr()], dtype=torch.int64, device=dev),
             torch.tensor([W.sm.data_ptr()], dtype=torch.int64, device=dev))
        _PTR_CACHE[key] = p
    return p


def _identity_off(T: int, dev):
    key = (T, str(dev))
    t = _OFF_CACHE.get(key)
    if t is None:
        t = torch.tensor([0, T], dtype=torch.int32, device=dev)
        _OFF_CACHE[key] = t
    return t


def _empty(dtype, dev):
    key = (dtype, str(dev))
    t = _EMPTY.get(key)
    if t is None:
        t = torch.empty(0, dtype=dtype, device=dev)
        _EMPTY[key] = t
    return t


def _EMPTY_I32(dev):
    return _empty(torch.int32, dev)


def _EMPTY_F32(dev):
    return _empty(torch.float32, dev)


def _EMPTY_BF16(dev):
    return _empty(torch.bfloat16, dev)


def block_sums(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """f32 sums of every 32-element block of each row of x (the min term of 4-bit GEMVs)."""
    ext().block_sums(x, out)
    _launched()
    return out


def moe_nt_hint(n_pairs: int, n_experts: int) -> int:
    """Token tiles of 8 per expert pass: sized for the mean load (an expert above it takes
    an extra pass over its weights, which is rarer than paying registers on every tile)."""
    mean = n_pairs / max(1, n_experts)
    return 1 if mean <= 4 else (2 if mean <= 10 else 4)


_STATUS: dict = {}


def gemm_status(dev) -> torch.Tensor:
    """Per-device int32 error word of the tcgen05 GEMM (bit 4: a pipeline wait timed out)."""
    key = str(dev)
    t = _STATUS.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _STATUS[key] = t
    return t


def gemm_grouped(x, qw_ptrs, sm_ptrs, row_off, N, K, mode, route_w, out, G, bank_qw=None, bank_sm=None):
    """tcgen05 GEMM over G contiguous row groups of x (bf16 [M, K]) with 4-bit weights.
    mode: 0 bf16 store, 1 SwiGLU, 2 f32 * route_w[row], 3 f32 +=, 5 f32 store.
    bank_qw/bank_sm: the contiguous weight bank (one matrix, or [G, ...] experts in group
    order) lets the kernel stream packed weights with 4-D TMA copies."""
    M = x.shape[0]
    if M == 0:
        return out
    max_mtiles = (M + 255) // 256 + G  # CTA tiles of 256 rows, at most one partial per group
    e = _EMPTY_I32(x.device)
    ext().tc_gemm_q4(x, qw_ptrs, sm_ptrs, row_off, N, K, mode,
                     route_w if route_w is not None else _EMPTY_F32(x.device), out, gemm_status(x.device),
                     max_mtiles, bank_qw if bank_qw is not None else e, bank_sm if bank_sm is not None else e, 0)
    _launched()
    return out


def gemm_grouped_banks(x, row_off, N, K, mode, route_w, out, banks, sel):
    """gemm_grouped over two contiguous weight banks streamed by TMA: banks = (q0, s0, q1, s1)
    with [entries, words] each; group g reads entry sel[g] >> 1 of bank sel[g] & 1."""
    M = x.shape[0]
    if M == 0:
        return out
    G = sel.numel()
    q0, s0, q1, s1 = banks
    ext().tc_gemm_q4_banks(x, row_off, N, K, mode, route_w if route_w is not None else _EMPTY_F32(x.device), out,
                           gemm_status(x.device), (M + 255) // 256 + G, q0, s0, q1, s1, sel)
    _launched()
    return out


def linear_grouped(x: torch.Tensor, bank, tok_off: torch.Tensor, tok_idx: torch.Tensor | None,
                   out: torch.Tensor, mode: int, route_w: torch.Tensor | None = None,
                   qw_ptrs: torch.Tensor | None = None, sm_ptrs: torch.Tensor | None = None,
                   nt_hint: int | None = None, xsum: torch.Tensor | None = None):
    """Grouped (per-expert) linear over CSR pair lists.  bank: ExpertBank (N, K, tensors)."""
    if x.is_cuda:
        e = ext()
        kmode = {GEMV_STORE: 0, GEMV_SWIGLU: 1, GEMV_SCALED_F32: 2}[mode]
        E = qw_ptrs.numel()
        if nt_hint is None:
            nt_hint = moe_nt_hint(out.shape[0], E)
        if getattr(bank, "is_fp8", False):
            xq, xs = e.f8_quant_act(x if x.stride(-1) == 1 else x.contiguous())
            e.f8_gemv(xq, xs, qw_ptrs, sm_ptrs, tok_off, tok_idx if tok_idx is not None else _EMPTY_I32(x.device),
                      route_w if route_w is not None else _EMPTY_F32(x.device), out, bank.N, bank.K, kmode, nt_hint,
                      _EMPTY_F32(x.device))
            _launched(2)
            return out
        e.q4_gemv(x, qw_ptrs, sm_ptrs, tok_off,
                  tok_idx if tok_idx is not None else _EMPTY_I32(x.device),
                  route_w if route_w is not None else _EMPTY_F32(x.device),
                  _EMPTY_BF16(x.device), out, bank.N, bank.K, kmode, nt_hint, min(E, out.shape[0]),
                  xsum if xsum is not None else _EMPTY_F32(x.device), bool(getattr(bank, "bank_contiguous", False)))
        _launched()
        return out
    # CPU reference: loop over experts in ascending order
    off = tok_off.tolist()
    for eidx in range(len(off) - 1):
        a, b = off[eidx], off[eidx + 1]
        if a == b:
            continue
        rows = tok_idx[a:b].long() if tok_idx is not None else torch.arange(a, b)
        y = x[rows].float() @ bank.weight(eidx).float().t()
        if mode == GEMV_SWIGLU:
            out[a:b] = swiglu_interleaved_ref(y)
        elif mode == GEMV_SCALED_F32:
            out[a:b] = route_w[a:b, None] * y
        else:
            out[a:b] = y
    return out


def qk_rope_kv_write(qkv, Hq, Hkv, D, q_norm, k_norm, eps, pos, cos_t, sin_t, slot, q_out, k_cache, v_cache):
    if qkv.is_cuda:
        ext().qk_rope_kv_write(qkv, Hq, Hkv, D, q_norm if q_norm is not None else _EMPTY_F32(qkv.device),
                               k_norm if k_norm is not None else _EMPTY_F32(qkv.device), eps, pos, cos_t, sin_t,
                               slot, q_out, k_cache, v_cache)
        _launched()
        return
    T = qkv.shape[0]
    x = qkv.float().reshape(T, Hq + 2 * Hkv, D)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]

    def _n(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w.float()

    if q_norm is not None:
        q = _n(q, q_norm)
        k = _n(k, k_norm)
    p = pos.long()
    c = cos_t[p][:, None, :]
    s = sin_t[p][:, None, :]

    def _r(t):
        a, b = t[..., : D // 2], t[..., D // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    q, k = _r(q), _r(k)
    q_out.copy_(q.reshape(q_out.shape))
    bs = k_cache.shape[2]
    for i in range(T):
        sl = int(slot[i])
        if sl < 0:
            continue
        k_cache[sl // bs, :, sl % bs] = k[i]
        v_cache[sl // bs, :, sl % bs] = v[i]


def attn_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, scale, part_o=None, part_ml=None,
                pages_per_split=16):
    """q: [T, Hq, D]; one query row per sequence, attending to ctx_lens[t] cached tokens."""
    if q.is_cuda:
        ext().attn_decode(q, k_cache, v_cache, block_tables, ctx_lens, part_o, part_ml, out, pages_per_split, scale)
        _launched(2)
        return out
    T, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    bs = k_cache.shape[2]
    for t in range(T):
        n = int(ctx_lens[t])
        nb = (n + bs - 1) // bs
        blocks = block_tables[t, :nb].long()
        k = k_cache[blocks].permute(0, 2, 1, 3).reshape(nb * bs, Hkv, D)[:n]
        v = v_cache[blocks].permute(0, 2, 1, 3).reshape(nb * bs, Hkv, D)[:n]
        g = Hq // Hkv
        kk = k.repeat_interleave(g, 1).float()
        vv = v.repeat_interleave(g, 1).float()
        s = torch.einsum("hd,khd->hk", q[t].float(), kk) * scale
        p = torch.softmax(s, -1)
        out[t] = torch.einsum("hk,khd->hd", p, vv).to(out.dtype)
    return out


def attn_prefill(q, k, v, cu_seqlens: list[int], out, scale):
    """Causal attention over freshly prefilled sequences (no cached prefix).
    q: [T, Hq, D], k/v: [T, Hkv, D] (rotated), out: [T, Hq, D]."""
    Hq, Hkv = q.shape[1], k.shape[1]
    for i in range(len(cu_seqlens) - 1):
        a, b = cu_seqlens[i], cu_seqlens[i + 1]
        qq = q[a:b].transpose(0, 1)[None]
        kk = k[a:b].transpose(0, 1)[None]
        vv = v[a:b].transpose(0, 1)[None]
        if not q.is_cuda:
            qq, kk, vv = qq.float(), kk.float(), vv.float()
        o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, scale=scale, enable_gqa=(Hq != Hkv))
        out[a:b] = o[0].transpose(0, 1).to(out.dtype)
    return out


# SYN_ATTN_TC: "1" (default) prefill attention on tcgen05, "0" the mma.sync kernel
_ATTN_TC = [__import__("os").environ.get("SYN_ATTN_TC", "1")]


def attn_prefill_paged(q, kc, vc, block_tables, cu_q, kv_lens, out, max_q_len: int, scale: float):
    """Causal prefill attention over the paged cache: query row i of sequence s (rows
    cu_q[s]..cu_q[s+1]) sits at position kv_lens[s] - q_len + i and attends to keys
    0..position through block_tables[s].  q/out: [T, Hq, D]; kc/vc: [blocks, Hkv, 16, D]."""
    if q.is_cuda and q.shape[-1] == 128:
        if _ATTN_TC[0] == "1":  # tcgen05 kernel (TMA-fed, S and P V in TMEM)
            ext().attn_prefill_tc(q, kc, vc, block_tables, cu_q, kv_lens, out, max_q_len, scale, gemm_status(q.device))
        else:                   # mma.sync kernel (the earlier tensor-core path, kept for comparison)
            ext().attn_prefill(q, kc, vc, block_tables, cu_q, kv_lens, out, max_q_len, scale)
        _launched()
        return out
    Hq, Hkv, D = q.shape[1], kc.shape[1], q.shape[2]
    cq, kl, bt = cu_q.tolist(), kv_lens.tolist(), block_tables.long()
    kflat = kc.permute(0, 2, 1, 3).reshape(-1, Hkv, D)
    vflat = vc.permute(0, 2, 1, 3).reshape(-1, Hkv, D)
    for s_idx in range(len(kl)):
        a, b, total = cq[s_idx], cq[s_idx + 1], kl[s_idx]
        n_new = b - a
        pos = torch.arange(total, device=q.device)
        sl = bt[s_idx][pos // 16] * 16 + pos % 16
        kk, vv = kflat[sl].transpose(0, 1)[None].float(), vflat[sl].transpose(0, 1)[None].float()
        qq = q[a:b].transpose(0, 1)[None].float()
        mask = pos[None, :] <= (torch.arange(n_new, device=q.device)[:, None] + (total - n_new))
        o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=scale, enable_gqa=(Hq != Hkv))
        out[a:b] = o[0].transpose(0, 1).to(out.dtype)
    return out


def mla_decode(q, cache, block_tables, ctx_lens, out, scale: float, part_o, part_ml, pages_per_split: int):
    """Absorbed MLA decode attention over the paged latent cache: q [B, H, 576] = [q_lat | q_pe]
    (bf16), cache [blocks, 16, 576]; out f32 [B, H, 512] = softmax(q . row) weighted latent rows."""
    ext().mla_decode(q, cache, block_tables, ctx_lens, out, scale, part_o, part_ml, pages_per_split)
    _launched(2)
    return out


def doorbell_wait(flag, want: int, timeout_s: float, status, waited_ns=None):
    """Bounded device wait until flag[0] >= want (sequence numbers); after timeout_s it sets
    bit 0 of status[0] and returns, leaving the context usable."""
    ext().doorbell_wait(flag, want, timeout_s, status,
                        waited_ns if waited_ns is not None else torch.empty(0, dtype=torch.int64, device=flag.device))
    _launched()


def doorbell_ring(flag, value: int):
    ext().doorbell_ring(flag, value)
    _launched()


def timestamp(buf, slot: int):
    """buf[slot] = device global timer (ns), in stream order."""
    ext().timestamp(buf, slot)
    _launched()


def tap_rows(x, idx, out):
    """Parity tap: out[i] = f32(x[idx[i]])."""
    if x.is_cuda:
        ext().tap_gather(x.contiguous(), idx, out)
        _launched()
    else:
        out.copy_(x[idx.long()].float())
    return out


def tap_compare(a, b):
    """Per-row (max |a-b|, ||a-b|| / ||b||) of two tap buffers, computed where they live."""
    if a.is_cuda:
        out = torch.empty(a.shape[0], 2, device=a.device)
        ext().tap_compare(a, b, out)
        _launched()
        return out
    d = (a - b).float()
    return torch.stack([d.abs().amax(-1), d.norm(dim=-1) / b.float().norm(dim=-1).clamp_min(1e-30)], -1)


def kv_pack(kc, vc, pages, packed=None):
    """K/V pages of a block list -> one contiguous buffer [n, 2, page] (offload, migration)."""
    page = kc[0].numel()
    if packed is None:
        packed = torch.empty(pages.numel(), 2, page, dtype=kc.dtype, device=kc.device)
    if kc.is_cuda:
        ext().kv_pages(kc, vc, pages, packed, True)
        _launched()
    else:
        packed[:, 0] = kc[pages.long()].reshape(pages.numel(), -1)
        packed[:, 1] = vc[pages.long()].reshape(pages.numel(), -1)
    return packed


def kv_unpack(packed, kc, vc, pages):
    """Inverse of kv_pack: writes the packed pages back into the caches at `pages`."""
    if kc.is_cuda:
        ext().kv_pages(kc, vc, pages, packed, False)
        _launched()
    else:
        kc[pages.long()] = packed[:, 0].reshape((pages.numel(),) + tuple(kc.shape[1:]))
        vc[pages.long()] = packed[:, 1].reshape((pages.numel(),) + tuple(vc.shape[1:]))


def router_logits(h, W, out):
    if h.is_cuda:
        ext().router_logits(h, W, out)
        _launched()
    else:
        out.copy_(h.float() @ W.float().t())
    return out


_TOPK_WS: dict = {}


def _topk_workspace(dev) -> torch.Tensor:
    """Zeroed int32 scratch of the routing kernel (token masks, prediction bits, arrival
    counter); every launch leaves it zeroed again.  One per device, kept for the process."""
    key = str(dev)
    ws = _TOPK_WS.get(key)
    if ws is None:
        ws = torch.zeros(4160, dtype=torch.int32, device=dev)
        _TOPK_WS[key] = ws
    return ws


def moe_topk(logits, cfg, bias, pred: bool, bufs: dict, counts=None, count_rows=None):
    """Top-k routing + CSR.  bufs: topk_ids, topk_w, tok_off, tok_idx, pair_w, pair_of, pred_mask.
    counts (int32 [E], optional) accumulates the number of pairs routed to each expert, over
    the rows t with count_rows[t] >= 0 when count_rows (int64 [T], e.g. the step slots) is given."""
    E, k = cfg.n_experts, cfg.top_k
    T = logits.shape[0]
    scoring = 0 if cfg.router_scoring == "softmax" else 1
    if logits.is_cuda:
        ext().moe_topk(logits, bias if bias is not None else _EMPTY_F32(logits.device), E, k, scoring, cfg.n_groups,
                       cfg.topk_groups, cfg.norm_topk_prob, cfg.routed_scaling, pred, bufs["topk_ids"],
                       bufs["topk_w"], bufs["tok_off"], bufs["tok_idx"], bufs["pair_w"], bufs["pair_of"],
                       bufs["pred_mask"] if pred else _EMPTY_I32(logits.device),
                       _topk_workspace(logits.device) if T <= 256 else
                       torch.zeros(E * ((T + 31) // 32) + E, dtype=torch.int32, device=logits.device),
                       counts if counts is not None else _EMPTY_I32(logits.device),
                       count_rows if count_rows is not None and counts is not None else _EMPTY_I32(logits.device))
        _launched()
        return
    from ..models.reference import topk_stable
    T = logits.shape[0]
    lg = logits[:, :E].float()
    if scoring == 0:
        scores = torch.softmax(lg, -1)
        sel = scores.clone()
    else:
        scores = torch.sigmoid(lg)
        sel = scores + (bias.float() if bias is not None else 0)
    if cfg.n_groups > 1:
        gs = sel.view(T, cfg.n_groups, E // cfg.n_groups)
        gscore = gs.topk(2, -1).values.sum(-1) if scoring == 1 else gs.max(-1).values
        _, gi = topk_stable(gscore, cfg.topk_groups)
        gm = torch.zeros_like(gscore).scatter_(1, gi, 1.0)
        sel = sel.masked_fill(gm[:, :, None].expand_as(gs).reshape(T, E) == 0, float("-inf"))
    _, ids = topk_stable(sel, k)
    w = torch.gather(scores, -1, ids)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    w = w * cfg.routed_scaling
    bufs["topk_ids"][:T] = ids.int()
    bufs["topk_w"][:T] = w
    n_e = torch.bincount(ids.reshape(-1), minlength=E)
    if counts is not None:
        live = ids if count_rows is None else ids[count_rows[:T].cpu() >= 0]
        counts[:E] += torch.bincount(live.reshape(-1), minlength=E).to(counts.dtype)
    off = torch.zeros(E + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(n_e, 0)
    bufs["tok_off"][: E + 1] = off.int()
    fill = off[:-1].clone()
    pair_of = torch.empty(T, k, dtype=torch.int32)
    for t in range(T):
        order = torch.argsort(ids[t])
        for slot, j in enumerate(order.tolist()):
            e = int(ids[t, j])
            p = int(fill[e])
            fill[e] += 1
            bufs["tok_idx"][p] = t
            bufs["pair_w"][p] = w[t, j]
            pair_of[t, slot] = p
    # pairs of one expert are in token order because tokens are visited in order
    bufs["pair_of"][:T] = pair_of


def moe_combine_rmsnorm(x, yp, pair_of, shared, w, out, eps):
    if x.is_cuda:
        ext().moe_combine_rmsnorm(x, yp, pair_of, shared if shared is not None else _EMPTY_F32(x.device),
                                  w if w is not None else _EMPTY_F32(x.device),
                                  out if out is not None else _EMPTY_BF16(x.device), eps)
        _launched()
        return
    T, k = pair_of.shape
    acc = torch.zeros_like(x)
    for j in range(k):
        acc += yp[pair_of[:, j].long()]
    if shared is not None:
        acc += shared
    x.add_(acc)
    if w is not None:
        out.copy_(rms_norm(x, w, eps))


def argmax(logits, out):
    if logits.is_cuda:
        ext().argmax(logits, out)
        _launched()
    else:
        out.copy_(torch.argmax(logits, -1).int())
    return out


def sample(logits, temperature, top_k, top_p, seed, stream, counter, out):
    if logits.is_cuda:
        ext().sample(logits, temperature, top_k, top_p, seed, stream, counter, out)
        _launched()
        return out
    from ..runtime.sampling_ref import sample_ref
    out.copy_(sample_ref(logits, temperature, top_k, top_p, seed, stream, counter))
    return out
