"""Kernel microbenchmarks at the flagship shapes (Qwen3-235B-A22B, batch 32 decode and
8192-token prefill).  Each kernel is timed with CUDA events after warm-up; inputs exceed
L2 (126 MB) wherever the kernel streams weights.  Reports achieved bandwidth / FLOP rate
as a fraction of the measured peaks in MEASURED_PEAKS.json (copy bandwidth, cuBLAS bf16).

    python -m syntropy_b200.bench.kernels [--only name,...]
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops
from .._ext import ext
from ..formats.q4 import Q4Weight

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def timeit(fn, iters=20, warmup=3, graph=True):
    """Device time per call (us).  The timed calls are captured in one CUDA graph and
    replayed, so host launch overhead does not show up in the number."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()  # warm
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
    else:
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


def bank(E, N, K, dev):
    from ..models.transformer import ExpertBank
    b = ExpertBank(E, N, K)
    b.qw = torch.empty(E, N * K // 8, dtype=torch.int32, device=dev)
    b.sm = torch.empty(E, N * K // 16, dtype=torch.float16, device=dev)
    for e in range(E):
        q = Q4Weight.quantize(torch.randn(N, K, device=dev) * 0.02)
        b.qw[e].copy_(q.qw)
        b.sm[e].copy_(q.sm)
    b.build_ptrs()
    return b


def routing(T, E, k, dev, seed=0):
    from ..models.config import get_config
    cfg = get_config("qwen3-235b-a22b").replace(n_experts=E, top_k=k)
    g = torch.Generator(device=dev).manual_seed(seed)
    logits = torch.randn(T, E, device=dev, generator=g)
    bufs = {"topk_ids": torch.zeros(T, k, dtype=torch.int32, device=dev),
            "topk_w": torch.zeros(T, k, device=dev), "tok_off": torch.zeros(E + 1, dtype=torch.int32, device=dev),
            "tok_idx": torch.zeros(T * k, dtype=torch.int32, device=dev), "pair_w": torch.zeros(T * k, device=dev),
            "pair_of": torch.zeros(T, k, dtype=torch.int32, device=dev), "pred_mask": None}
    ops.moe_topk(logits, cfg, None, False, bufs)
    return cfg, bufs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--dense", default="", help="extra dense GEMV shapes 'N:K,N:K' (e.g. Llama-3-70B layers)")
    args = ap.parse_args()
    only = set(x for x in args.only.split(",") if x)
    dev = torch.device("cuda:0")
    hbm, tf, src = peaks()
    res = []
    T = args.batch

    def report(name, us, nbytes=None, flops=None, extra=None):
        r = {"kernel": name, "us": round(us, 2)}
        if nbytes:
            r["GB/s"] = round(nbytes / us / 1e3, 1)
            r["frac_hbm"] = round(nbytes / us / 1e3 / hbm, 3)
        if flops:
            r["TFLOP/s"] = round(flops / us / 1e6, 1)
            r["frac_bf16"] = round(flops / us / 1e6 / tf, 3)
        if extra:
            r.update(extra)
        r["peak_source"] = src
        res.append(r)
        print(json.dumps(r), flush=True)

    want = lambda n: not only or n in only  # noqa: E731
    H, f, E, k = 4096, 1536, 128, 8
    if want("moe_gate_up") or want("moe_down"):
        cfg, b = routing(T, E, k, dev)
        gu = bank(E, 2 * f, H, dev)
        dn = bank(E, H, f, dev)
        h = torch.randn(T, H, device=dev).to(torch.bfloat16)
        mid = torch.empty(T * k, f, dtype=torch.bfloat16, device=dev)
        yp = torch.empty(T * k, H, dtype=torch.float32, device=dev)
        active = int((b["tok_off"][1:] - b["tok_off"][:-1] > 0).sum())
        fn = lambda: ops.linear_grouped(h, gu, b["tok_off"], b["tok_idx"], mid, ops.GEMV_SWIGLU,  # noqa: E731
                                        qw_ptrs=gu.qw_ptrs, sm_ptrs=gu.sm_ptrs)
        report("moe_gate_up_gemv", timeit(fn), active * gu.N * gu.K * 5 // 8, extra={"active_experts": active})
        xs = torch.empty(T, H // 32, device=dev)

        def fn_pre():
            ops.block_sums(h, xs)
            ops.linear_grouped(h, gu, b["tok_off"], b["tok_idx"], mid, ops.GEMV_SWIGLU, qw_ptrs=gu.qw_ptrs,
                               sm_ptrs=gu.sm_ptrs, xsum=xs)
        report("moe_gate_up_gemv+block_sums", timeit(fn_pre), active * gu.N * gu.K * 5 // 8)
        fn = lambda: ops.linear_grouped(mid, dn, b["tok_off"], None, yp, ops.GEMV_SCALED_F32,  # noqa: E731
                                        route_w=b["pair_w"], qw_ptrs=dn.qw_ptrs, sm_ptrs=dn.sm_ptrs)
        report("moe_down_gemv", timeit(fn), active * dn.N * dn.K * 5 // 8, extra={"active_experts": active})
        del gu, dn
    extra = [(f"dense_{n}x{k}", int(n), int(k)) for n, k in (x.split(":") for x in args.dense.split(",") if x)]
    for name, N, K in [("qkv_gemv", 9216, 4096), ("o_gemv", 4096, 8192), ("lm_head_gemv", 151936, 4096)] + extra:
        if not want(name) and not name.startswith("dense_"):
            continue
        reps = max(1, int(math.ceil(300e6 / (N * K * 5 / 8))))  # rotate copies to exceed L2
        ws = [Q4Weight.quantize(torch.randn(N, K, device=dev) * 0.02) for _ in range(reps)]
        x = torch.randn(T, K, device=dev).to(torch.bfloat16)
        out = torch.empty(T, N, dtype=torch.float32 if name == "lm_head_gemv" else torch.bfloat16, device=dev)
        i = [0]

        def fn():
            ops.linear(x, ws[i[0] % reps], out, ops.GEMV_STORE)
            i[0] += 1
        report(name, timeit(fn, warmup=max(3, reps)), N * K * 5 // 8)
        del ws
    if want("router"):
        W = (torch.randn(2 * E, H, device=dev) * 0.02).to(torch.bfloat16)
        h = torch.randn(T, H, device=dev).to(torch.bfloat16)
        lg = torch.empty(T, 2 * E, device=dev)
        report("router_logits", timeit(lambda: ops.router_logits(h, W, lg)), W.numel() * 2)
        cfg, b = routing(T, E, k, dev)
        b["pred_mask"] = torch.zeros(E, dtype=torch.int32, device=dev)
        report("moe_topk", timeit(lambda: ops.moe_topk(lg, cfg, None, True, b)))
    if want("attn"):
        from ..kv.paged import PagedKVCache
        ctx, Hq, Hkv, D = 1024, 64, 4, 128
        nb = T * (ctx // 16) + 1
        kc = torch.randn(nb, Hkv, 16, D, device=dev).to(torch.bfloat16)
        vc = torch.randn(nb, Hkv, 16, D, device=dev).to(torch.bfloat16)
        bt = (torch.randperm(nb - 1, device=dev)[: T * (ctx // 16)] + 1).int().view(T, -1)
        cl = torch.full((T,), ctx, dtype=torch.int32, device=dev)
        q = torch.randn(T, Hq, D, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        for pps in (16, 8, 4):  # pages per KV split: CTAs = T x Hkv x splits (16: the runner's default)
            ns = (bt.shape[1] + pps - 1) // pps
            po = torch.empty(T * Hkv * ns * 16 * D, device=dev)
            pml = torch.empty(T * Hkv * ns * 16 * 2, device=dev)
            fn = lambda: ops.attn_decode(q, kc, vc, bt, cl, out, 1 / math.sqrt(D), po, pml, pps)  # noqa: E731
            report("attn_decode" if pps == 16 else f"attn_decode_pps{pps}", timeit(fn), T * ctx * Hkv * D * 2 * 2)
    if want("gemm_tc"):
        for M, N, K in ((8192, 9216, 4096), (8192, 4096, 8192)):
            w = Q4Weight.quantize(torch.randn(N, K, device=dev) * 0.02)
            x = torch.randn(M, K, device=dev).to(torch.bfloat16)
            out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            st = torch.zeros(1, dtype=torch.int32, device=dev)
            qp = torch.tensor([w.qw.data_ptr()], device=dev)
            sp = torch.tensor([w.sm.data_ptr()], device=dev)
            off = torch.tensor([0, M], dtype=torch.int32, device=dev)
            fn = lambda: ext().tc_gemm_q4(x, qp, sp, off, N, K, 0, torch.empty(0, device=dev), out, st,  # noqa: E731
                                          M // 128 + 1, w.qw, w.sm, 0)
            report(f"tc_gemm_q4_{M}x{N}x{K}", timeit(fn, iters=10), flops=2 * M * N * K,
                   extra={"status": int(st.item())})
            wd = w.dequant()
            report(f"cublas_bf16_{M}x{N}x{K}(reference)", timeit(lambda: x @ wd.t(), iters=10), flops=2 * M * N * K)
    if want("q4_dec") or "q4_dec_small" in only:
        # 4-bit weights at 16-64 decode rows (Llama-3-70B layer shapes, one GPU and one TP8 rank):
        # the tcgen05 decode GEMM against the mma.sync GEMV on the same inputs; weights in
        # rotated copies larger than L2
        from syntropy_b200.ops import core as _core
        # q4_dec_small: one shape at 32 rows (a profiler-sized case)
        small = "q4_dec_small" in only
        shapes = ((8192, 8192),) if small else ((10240, 8192), (8192, 8192), (57344, 8192), (8192, 28672),
                                                (1280, 8192), (7168, 8192), (8192, 3584))
        for N, K in shapes:
            ncopy = max(1, int(2 * 126e6 // (N * K // 2)) + 1)
            ws = [Q4Weight.quantize(torch.randn(N, K, device=dev) * 0.02) for _ in range(min(ncopy, 64))]
            for rows in ((32,) if small else (16, 32, 64)):
                x = torch.randn(rows, K, device=dev).to(torch.bfloat16)
                out = torch.empty(rows, N, dtype=torch.float32, device=dev)
                it = [0]

                def fn():
                    it[0] += 1
                    ops.linear(x, ws[it[0] % len(ws)], out, ops.GEMV_STORE)
                nbytes = N * K // 2 + N * K // 8
                saved = _core._Q4_TC[0]
                for impl, thr in (("tcgen05", 16), ("mma_sync_gemv", 1 << 30)):
                    _core._Q4_TC[0] = thr
                    # warm-up touches every copy (per-weight pointer tables are built outside capture)
                    report(f"q4_dec_{impl}_{rows}x{N}x{K}", timeit(fn, iters=20, warmup=len(ws) + 2), nbytes=nbytes,
                           flops=2 * rows * N * K)
                _core._Q4_TC[0] = saved
    if want("moe_prefill") or "moe_prefill_small" in only:
        # grouped 4-bit GEMMs of one Qwen3-235B MoE layer over a 32768-token prefill pass
        # (top-8 of 128 experts: ~2048 rows per expert), all experts in one contiguous bank;
        # moe_prefill_small: 16 experts (a profiler-sized case)
        G, rows_per = (16 if "moe_prefill_small" in only else 128), 2048
        off = torch.arange(0, (G + 1) * rows_per, rows_per, dtype=torch.int32, device=dev)
        M = G * rows_per
        for name, N, K in (("gate_up", 3072, 4096), ("down", 4096, 1536)):
            wq = [Q4Weight.quantize(torch.randn(N, K, device=dev) * 0.02) for _ in range(4)]
            qb = torch.stack([wq[e % 4].qw for e in range(G)])
            sb = torch.stack([wq[e % 4].sm for e in range(G)])
            qp = torch.tensor([qb[e].data_ptr() for e in range(G)], dtype=torch.int64, device=dev)
            sp = torch.tensor([sb[e].data_ptr() for e in range(G)], dtype=torch.int64, device=dev)
            x = torch.randn(M, K, device=dev).to(torch.bfloat16)
            out = torch.empty(M, N // 2 if name == "gate_up" else N,
                              dtype=torch.bfloat16 if name == "gate_up" else torch.float32, device=dev)
            rw = torch.rand(M, device=dev)
            mode = 1 if name == "gate_up" else 2
            report(f"moe_prefill_{name}_{G}x{rows_per}x{N}x{K}",
                   timeit(lambda: ops.gemm_grouped(x, qp, sp, off, N, K, mode, rw, out, G, qb, sb), iters=5),
                   flops=2 * M * N * K)
            del qb, sb, x, out
    if want("gemm_bf16"):
        # Llama-3-8B bf16 projections: one GPU and one TP8 rank at decode (64 rows), and a
        # 2048-token prefill; our tcgen05 GEMM against the library GEMM on the same inputs
        shapes = [("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336),
                  ("tp8_qkv", 768, 4096), ("tp8_o", 4096, 512), ("tp8_gate_up", 3584, 4096),
                  ("tp8_down", 4096, 1792)]
        from ..ops.core import _bf16_workspace, gemm_status
        for rows in (T, 2048):
            for name, N, K in shapes:
                if rows > 256 and name.startswith("tp8"):
                    continue
                reps = max(1, int(math.ceil(300e6 / (N * K * 2)))) if rows <= 256 else 1
                wl = [(torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16) for _ in range(reps)]
                x = torch.randn(rows, K, device=dev).to(torch.bfloat16)
                out = torch.empty(rows, N, dtype=torch.bfloat16, device=dev)
                ws, ctr = _bf16_workspace(dev, N, K, rows)
                st = gemm_status(dev)
                i = [0]

                def fnb():
                    ext().gemm_bf16(x, wl[i[0] % reps], out, 0, ws, ctr, st)
                    i[0] += 1

                def fnl():
                    torch.matmul(x, wl[i[0] % reps].t(), out=out)
                    i[0] += 1
                nb, fl = N * K * 2, 2 * rows * N * K
                tag = f"{name}_{rows}x{N}x{K}"
                report(f"gemm_bf16_tc_{tag}", timeit(fnb, warmup=max(3, reps), iters=max(20, reps)), nb, fl,
                       extra={"splits": ext().gemm_bf16_ws(N, K, rows) and None})
                report(f"gemm_bf16_library_{tag}(reference)", timeit(fnl, warmup=max(3, reps), iters=max(20, reps)),
                       nb, fl)
                del wl
    if want("fp8_gemv"):
        from ..formats.fp8 import FP8Weight
        for name, N, K, rows in (("fp8_gemv_dense_7168x18432", 7168, 18432, T), ("fp8_lm_head_129280x7168", 129280, 7168, 2)):
            reps = max(1, int(math.ceil(300e6 / (N * K))))
            ws = [FP8Weight.quantize(torch.randn(N, K, device=dev) * 0.02) for _ in range(reps)]
            x = torch.randn(rows, K, device=dev).to(torch.bfloat16)
            out = torch.empty(rows, N, dtype=torch.float32, device=dev)
            i = [0]

            def fn8():
                ops.linear(x, ws[i[0] % reps], out, ops.GEMV_STORE)
                i[0] += 1
            report(name, timeit(fn8, warmup=max(3, reps)), N * K + (N // 128 + 1) * (K // 128) * 4,
                   extra={"rows": rows})
            del ws
    if want("mla"):
        B, H, ctx = 16, 128, 4096
        nb = B * ctx // 16 + 1
        cache = torch.randn(nb, 16, 576, device=dev).to(torch.bfloat16)
        bt = (torch.randperm(nb - 1, device=dev)[: B * ctx // 16] + 1).int().view(B, -1)
        cl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
        q = torch.randn(B, H, 576, device=dev).to(torch.bfloat16)
        pps = 32
        ns = (bt.shape[1] + pps - 1) // pps
        po = torch.empty(B * H * ns * 512, device=dev)
        pml = torch.empty(B * H * ns * 2, device=dev)
        o = torch.empty(B, H, 512, device=dev)
        report("mla_decode_b16_ctx4096", timeit(lambda: ops.mla_decode(q, cache, bt, cl, o, 1 / math.sqrt(192), po, pml,
                                                                       pps)), B * ctx * 1152)
    if want("attn_prefill") or "attn_prefill_small" in only:
        import torch.nn.functional as F
        from syntropy_b200.ops import core as _core
        # Qwen3-235B prompt shape (8 x 1024, 64 q / 4 kv heads) and Llama-3-8B (4 x 2048, 32 / 8);
        # attn_prefill_small: one 4 x 1024 (32 / 8) case, small enough for a profiler capture
        shapes = ((4, 1024, 32, 8),) if "attn_prefill_small" in only else ((8, 1024, 64, 4), (4, 2048, 32, 8))
        for nseq, L, Hq, Hkv in shapes:
            D = 128
            nb = nseq * L // 16 + 1
            kc = torch.randn(nb, Hkv, 16, D, device=dev).to(torch.bfloat16)
            vc = torch.randn(nb, Hkv, 16, D, device=dev).to(torch.bfloat16)
            bt = (torch.arange(nseq * L // 16, device=dev) + 1).int().view(nseq, -1)
            cu = torch.arange(0, nseq * L + 1, L, dtype=torch.int32, device=dev)
            kl = torch.full((nseq,), L, dtype=torch.int32, device=dev)
            q = torch.randn(nseq * L, Hq, D, device=dev).to(torch.bfloat16)
            o = torch.empty_like(q)
            flops = 4 * nseq * L * L * Hq * D / 2  # causal
            tag = f"{nseq}x{L}_h{Hq}kv{Hkv}"
            saved = _core._ATTN_TC[0]
            for impl, flag in (("tcgen05", "1"), ("mma_sync", "0")):
                _core._ATTN_TC[0] = flag
                report(f"attn_prefill_{impl}_{tag}",
                       timeit(lambda: ops.attn_prefill_paged(q, kc, vc, bt, cu, kl, o, L, 1 / math.sqrt(D)),
                              iters=10), flops=flops)
            _core._ATTN_TC[0] = saved
            qq = q.view(nseq, L, Hq, D).transpose(1, 2)
            kk = kc[1:].permute(0, 2, 1, 3).reshape(nseq, L, Hkv, D).transpose(1, 2)
            vv = vc[1:].permute(0, 2, 1, 3).reshape(nseq, L, Hkv, D).transpose(1, 2)
            report(f"sdpa_library_{tag}(reference)",
                   timeit(lambda: F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=True),
                          iters=10), flops=flops)
    print(json.dumps({"summary": res}))


if __name__ == "__main__":
    main()
