"""sm_100a kernels against plain f32 PyTorch references of the same op."""
import math

import pytest
import torch

from syntropy_b200 import ops
from syntropy_b200._ext import ext
from syntropy_b200.formats.q4 import Q4Weight, dequant_rows_ref
from syntropy_b200.models.config import get_config
from syntropy_b200.runtime.sampling_ref import sample_ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def test_q4_quantize_matches_cpu_oracle(cuda):
    w = torch.randn(128, 512) * 0.02
    rows_cpu = ext().q4_quantize_rows_cpu(w)
    q = Q4Weight.quantize(w.to(cuda))
    assert torch.equal(q.to_rows().cpu(), rows_cpu)
    deq = q.dequant().float().cpu()
    ref = dequant_rows_ref(rows_cpu, 128, 512)
    assert torch.allclose(deq, ref.to(torch.bfloat16).float(), atol=0, rtol=0)
    q2 = Q4Weight.from_rows(rows_cpu.to(cuda), 128, 512)
    assert torch.equal(q2.qw, q.qw) and torch.equal(q2.sm, q.sm)


@pytest.fixture
def gemv_only():
    """Keep 32-64-row 4-bit products on the mma.sync GEMV (its exact f32 scale/min fold is what
    these tests check; the tcgen05 decode GEMM has its own tests)."""
    from syntropy_b200.ops import core
    saved = core._Q4_TC[0]
    core._Q4_TC[0] = 1 << 30
    yield
    core._Q4_TC[0] = saved


@pytest.mark.parametrize("T,N,K", [(1, 256, 512), (5, 512, 1024), (8, 4096, 4096), (32, 1024, 4096),
                                   (64, 256, 1536), (3, 9216, 4096)])
def test_q4_gemv_dense(cuda, gemv_only, T, N, K):
    torch.manual_seed(0)
    w = torch.randn(N, K, device=cuda) * 0.02
    q = Q4Weight.quantize(w)
    wd = ext().q4t_dequant(q.qw, q.sm, N, K)  # bf16 (exact for these magnitudes? compare vs f32 dequant below)
    rows = q.to_rows().cpu()
    wf = dequant_rows_ref(rows, N, K).to(cuda)
    x = (torch.randn(T, K, device=cuda)).to(torch.bfloat16)
    out = torch.empty(T, N, dtype=torch.bfloat16, device=cuda)
    ops.linear(x, q, out, ops.GEMV_STORE)
    ref = x.float() @ wf.t()
    assert _rel(out, ref) < 4e-3
    # f32 residual epilogue
    res = torch.randn(T, N, device=cuda)
    r0 = res.clone()
    ops.linear(x, q, res, ops.GEMV_ADD_F32)
    assert _rel(res - r0, ref) < 1e-4
    del wd


def test_q4_gemv_grouped_swiglu_and_scaled(cuda):
    torch.manual_seed(1)
    E, f, H, T, k = 8, 256, 512, 6, 3
    g = torch.randn(E, f, H, device=cuda) * 0.02
    u = torch.randn(E, f, H, device=cuda) * 0.02
    d = torch.randn(E, H, f, device=cuda) * 0.02
    from syntropy_b200.models.transformer import ExpertBank
    gu = ExpertBank(E, 2 * f, H)
    dn = ExpertBank(E, H, f)
    gu.qw = torch.zeros(E, 2 * f * H // 8, dtype=torch.int32, device=cuda)
    gu.sm = torch.zeros(E, 2 * f * H // 16, dtype=torch.float16, device=cuda)
    dn.qw = torch.zeros(E, H * f // 8, dtype=torch.int32, device=cuda)
    dn.sm = torch.zeros(E, H * f // 16, dtype=torch.float16, device=cuda)
    for e in range(E):
        q = Q4Weight.quantize(ops.interleave_gate_up(g[e], u[e]))
        gu.qw[e].copy_(q.qw); gu.sm[e].copy_(q.sm)
        q = Q4Weight.quantize(d[e])
        dn.qw[e].copy_(q.qw); dn.sm[e].copy_(q.sm)
    gu.build_ptrs(); dn.build_ptrs()
    cfg = get_config("tiny-qwen-moe").replace(n_experts=E, top_k=k, hidden=H, moe_ffn=f)
    h = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    logits = torch.randn(T, E, device=cuda)
    bufs = {"topk_ids": torch.zeros(T, k, dtype=torch.int32, device=cuda),
            "topk_w": torch.zeros(T, k, device=cuda), "tok_off": torch.zeros(E + 1, dtype=torch.int32, device=cuda),
            "tok_idx": torch.zeros(T * k, dtype=torch.int32, device=cuda), "pair_w": torch.zeros(T * k, device=cuda),
            "pair_of": torch.zeros(T, k, dtype=torch.int32, device=cuda), "pred_mask": None}
    ops.moe_topk(logits, cfg, None, False, bufs)
    mid = torch.empty(T * k, f, dtype=torch.bfloat16, device=cuda)
    ops.linear_grouped(h, gu, bufs["tok_off"], bufs["tok_idx"], mid, ops.GEMV_SWIGLU, qw_ptrs=gu.qw_ptrs,
                       sm_ptrs=gu.sm_ptrs)
    yp = torch.empty(T * k, H, device=cuda)
    ops.linear_grouped(mid, dn, bufs["tok_off"], None, yp, ops.GEMV_SCALED_F32, route_w=bufs["pair_w"],
                       qw_ptrs=dn.qw_ptrs, sm_ptrs=dn.sm_ptrs)
    x = torch.zeros(T, H, device=cuda)
    ops.moe_combine_rmsnorm(x, yp, bufs["pair_of"], None, None, None, 1e-6)
    # reference in f32 with dequantised weights
    ref = torch.zeros(T, H, device=cuda)
    for t in range(T):
        for j in range(k):
            e = int(bufs["topk_ids"][t, j])
            wg = gu.weight(e).float()
            a = ops.swiglu_interleaved_ref(h[t:t + 1].float() @ wg.t())
            ref[t] += bufs["topk_w"][t, j] * (a.to(torch.bfloat16).float() @ dn.weight(e).float().t())[0]
    assert _rel(x, ref) < 1e-2


@pytest.mark.parametrize("T", [32, 3, 256, 700])
def test_moe_topk_matches_cpu(cuda, T):
    torch.manual_seed(2)
    cfg = get_config("qwen3-235b-a22b")
    E, k = cfg.n_experts, cfg.top_k
    pred_on = T <= 256  # next-layer prediction is a decode-size feature
    logits = torch.randn(T, 2 * E if pred_on else E)

    def bufs(dev):
        return {"topk_ids": torch.zeros(T, k, dtype=torch.int32, device=dev),
                "topk_w": torch.zeros(T, k, device=dev), "tok_off": torch.zeros(E + 1, dtype=torch.int32, device=dev),
                "tok_idx": torch.zeros(T * k, dtype=torch.int32, device=dev), "pair_w": torch.zeros(T * k, device=dev),
                "pair_of": torch.zeros(T, k, dtype=torch.int32, device=dev),
                "pred_mask": torch.zeros(E, dtype=torch.int32, device=dev)}

    bc, bg = bufs("cpu"), bufs(cuda)
    ops.moe_topk(logits[:, :E].contiguous(), cfg, None, False, bc)
    counts = torch.zeros(E, dtype=torch.int32, device=cuda)
    # usage counts: decode batches skip rows marked -1 (bucket padding); prefill counts all
    rows = torch.where(torch.arange(T) % 5 == 4, -1, 1) if pred_on else None
    for _ in range(2):  # the second call checks that the kernel left its workspace zeroed
        ops.moe_topk(logits.to(cuda), cfg, None, pred_on, bg, counts=counts,
                     count_rows=rows.to(cuda) if rows is not None else None)
        for key in ("topk_ids", "tok_off", "tok_idx", "pair_of"):
            assert torch.equal(bc[key], bg[key].cpu()), key
        assert torch.allclose(bc["topk_w"], bg["topk_w"].cpu(), rtol=1e-5, atol=1e-6)
        assert torch.allclose(bc["pair_w"], bg["pair_w"].cpu(), rtol=1e-5, atol=1e-6)
    live = bc["topk_ids"] if rows is None else bc["topk_ids"][rows >= 0]
    assert torch.equal(counts.cpu(), 2 * torch.bincount(live.reshape(-1).long(), minlength=E).int())
    if not pred_on:
        return
    # prediction mask = union of the next layer's top-k
    pred = torch.zeros(E, dtype=torch.int32)
    pred[torch.sort(-torch.softmax(logits[:, E:], -1), dim=-1, stable=True).indices[:, :k].reshape(-1)] = 1
    assert torch.equal(pred, bg["pred_mask"].cpu())


def test_deepseek_group_routing_matches_cpu(cuda):
    torch.manual_seed(3)
    cfg = get_config("deepseek-v3")
    E, k, T = cfg.n_experts, cfg.top_k, 16
    logits = torch.randn(T, E)
    bias = torch.randn(E) * 0.1

    def bufs(dev):
        return {"topk_ids": torch.zeros(T, k, dtype=torch.int32, device=dev),
                "topk_w": torch.zeros(T, k, device=dev), "tok_off": torch.zeros(E + 1, dtype=torch.int32, device=dev),
                "tok_idx": torch.zeros(T * k, dtype=torch.int32, device=dev), "pair_w": torch.zeros(T * k, device=dev),
                "pair_of": torch.zeros(T, k, dtype=torch.int32, device=dev), "pred_mask": None}

    bc, bg = bufs("cpu"), bufs(cuda)
    ops.moe_topk(logits, cfg, bias, False, bc)
    ops.moe_topk(logits.to(cuda), cfg, bias.to(cuda), False, bg)
    assert torch.equal(torch.sort(bc["topk_ids"], -1).values, torch.sort(bg["topk_ids"].cpu(), -1).values)
    assert torch.allclose(bc["topk_w"].sort(-1).values, bg["topk_w"].cpu().sort(-1).values, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("G,D,ctx", [(16, 128, [1, 17, 300, 1025]), (4, 128, [33, 64, 5]), (8, 128, [700])])
def test_attn_decode(cuda, G, D, ctx):
    torch.manual_seed(4)
    Hkv = 2
    Hq = G * Hkv
    T = len(ctx)
    bs = 16
    maxb = max((c + bs - 1) // bs for c in ctx)
    nblocks = T * maxb + 1
    kc = torch.randn(nblocks, Hkv, bs, D, device=cuda).to(torch.bfloat16)
    vc = torch.randn(nblocks, Hkv, bs, D, device=cuda).to(torch.bfloat16)
    perm = torch.randperm(nblocks - 1) + 1
    bt = perm[: T * maxb].view(T, maxb).to(torch.int32).to(cuda)
    q = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    cl = torch.tensor(ctx, dtype=torch.int32, device=cuda)
    out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=cuda)
    pps = 4
    ns = (maxb + pps - 1) // pps
    po = torch.empty(T * Hkv * ns * 16 * D, device=cuda)
    pml = torch.empty(T * Hkv * ns * 16 * 2, device=cuda)
    ops.attn_decode(q, kc, vc, bt, cl, out, 1 / math.sqrt(D), po, pml, pps)
    ref = torch.empty(T, Hq, D)
    ops.attn_decode(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), bt.cpu(), cl.cpu(), ref, 1 / math.sqrt(D))
    assert _rel(out.cpu(), ref) < 1e-2


def test_qk_rope_kv_write(cuda):
    torch.manual_seed(5)
    Hq, Hkv, D, T = 8, 2, 128, 7
    from syntropy_b200.models.reference import rope_table
    cos, sin = rope_table(D, 1e6, 4096)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 5, 100, 2000, 3, 4095], dtype=torch.int32)
    slot = torch.tensor([16, 17, 40, 3, 90, -1, 5], dtype=torch.int64)
    qn, kn = torch.rand(D) + 0.5, torch.rand(D) + 0.5
    kc = torch.zeros(8, Hkv, 16, D)
    vc = torch.zeros(8, Hkv, 16, D)
    qo = torch.zeros(T, Hq, D)
    ops.qk_rope_kv_write(qkv.float(), Hq, Hkv, D, qn, kn, 1e-6, pos, cos, sin, slot, qo, kc, vc)
    kg, vg = kc.to(torch.bfloat16).to(cuda) * 0, vc.to(torch.bfloat16).to(cuda) * 0
    qg = torch.zeros(T, Hq, D, dtype=torch.bfloat16, device=cuda)
    ops.qk_rope_kv_write(qkv.to(cuda), Hq, Hkv, D, qn.to(cuda), kn.to(cuda), 1e-6, pos.to(cuda), cos.to(cuda),
                         sin.to(cuda), slot.to(cuda), qg, kg, vg)
    assert _rel(qg.cpu(), qo) < 5e-3
    assert _rel(kg.cpu(), kc) < 5e-3
    assert _rel(vg.cpu(), vc) < 5e-3


def test_sampler(cuda):
    torch.manual_seed(6)
    T, V = 16, 151936
    logits = torch.randn(T, V) * 3
    # Philox device == host
    assert torch.equal(ext().philox(123, 7, 1000, 4096, logits.to(cuda)).cpu(), ext().philox_cpu(123, 7, 1000, 4096))
    temp = torch.tensor([0.0] * 4 + [1.0] * 12)
    topk = torch.tensor([0] * 8 + [50] * 4 + [0] * 4, dtype=torch.int32)
    topp = torch.tensor([1.0] * 12 + [0.9] * 4)
    seed = torch.arange(T, dtype=torch.int64) * 7919
    stream = torch.arange(T, dtype=torch.int64)
    ctr = torch.zeros(T, dtype=torch.int64)
    out = torch.empty(T, dtype=torch.int32, device=cuda)
    ctr_g = ctr.to(cuda)
    ops.sample(logits.to(cuda), temp.to(cuda), topk.to(cuda), topp.to(cuda), seed.to(cuda), stream.to(cuda), ctr_g,
               out)
    ref = sample_ref(logits, temp, topk, topp, seed, stream, ctr.clone())
    assert torch.equal(out.cpu()[:4], torch.argmax(logits[:4], -1).int())
    # Both sides draw the same Philox number and select by the same fixed-point inverse CDF;
    # the masses exp(z - max) * 2^32 come from the device's fast exp and the host's exp, which
    # agree to a few ulp, not bit for bit.  So the tokens must be equal, except where the
    # draw's target lands within that rounding distance of a cumulative boundary, where the
    # two picks may be neighbours in the CDF.  Each such row is checked for exactly that.
    from syntropy_b200.runtime.sampling_ref import _row_masses, philox_draw
    dev = out.cpu()
    for t in range(4, T):
        if int(dev[t]) == int(ref[t]):
            continue
        mass = _row_masses(logits[t], float(temp[t]), int(topk[t]), float(topp[t])).double()
        total = float(mass.sum())
        target = (philox_draw(int(seed[t]), int(stream[t]), 0) * int(mass.sum())) >> 32
        cum = torch.cumsum(mass, 0)
        lo, hi = sorted((int(dev[t]), int(ref[t])))
        boundary = float(cum[lo])  # the boundary between the two picks
        assert float(mass[lo + 1:hi].sum()) == 0.0, (t, dev[t], ref[t])  # neighbours in the CDF
        assert abs(target - boundary) <= 1e-5 * total, (t, dev[t], ref[t], target, boundary)
    assert torch.equal(ctr_g.cpu(), (temp > 0).long())


@pytest.mark.parametrize("T,N,K,mode", [(32, 9216, 4096, 0), (16, 4096, 8192, 3), (24, 3072, 4096, 1),
                                         (64, 1024, 1536, 5), (9, 4096, 4096, 0)])
def test_q4_gemv_dense_splitk(cuda, gemv_only, T, N, K, mode):
    torch.manual_seed(7)
    w = torch.randn(N, K, device=cuda) * 0.02
    q = Q4Weight.quantize(w)
    wf = dequant_rows_ref(q.to_rows().cpu(), N, K).to(cuda)
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    ref = x.float() @ wf.t()
    if mode == 1:
        out = torch.empty(T, N // 2, dtype=torch.bfloat16, device=cuda)
        ops.linear(x, q, out, ops.GEMV_SWIGLU)
        assert _rel(out, ops.swiglu_interleaved_ref(ref)) < 1e-2
    elif mode == 3:
        out = torch.randn(T, N, device=cuda)
        o0 = out.clone()
        ops.linear(x, q, out, ops.GEMV_ADD_F32)
        assert _rel(out - o0, ref) < 1e-4
    else:
        out = torch.empty(T, N, dtype=torch.bfloat16 if mode == 0 else torch.float32, device=cuda)
        ops.linear(x, q, out, ops.GEMV_STORE)
        assert _rel(out, ref) < (4e-3 if mode == 0 else 1e-4)
    # deterministic: a second call gives identical bits
    out2 = out.clone()
    if mode != 3:
        ops.linear(x, q, out2, ops.GEMV_SWIGLU if mode == 1 else ops.GEMV_STORE)
        assert torch.equal(out, out2)


@pytest.mark.parametrize("stochastic", [False, True])
def test_verify_accept_matches_host_oracle(cuda, stochastic):
    """Device VerifyAccept against its host oracle, bit for bit: tokens, accepted counts and
    Philox counters, for greedy and sampled rows (top-k / top-p included), with point-mass or
    stochastic drafts (the drafts' own distributions given)."""
    from syntropy_b200.runtime.sampling_ref import verify_ref
    from syntropy_b200.runtime.spec import verify
    torch.manual_seed(5)
    S, g, V = 12, 3, 5000
    logits = torch.randn(S * (g + 1), V) * 3
    q = torch.softmax(torch.randn(S, g, V) * 2, -1) if stochastic else None
    drafts = torch.stack([torch.multinomial(q[s], 1)[:, 0] for s in range(S)]).int() if stochastic else \
        torch.randint(0, V, (S, g), dtype=torch.int32)
    # make some drafts the target's argmax so that acceptance paths run too
    for s in range(0, S, 3):
        drafts[s, 0] = int(logits[s * (g + 1)].argmax())
    temp = torch.tensor([0.0, 0.8, 1.0, 1.3] * (S // 4))
    top_k = torch.tensor([0, 0, 50, 0] * (S // 4), dtype=torch.int32)
    top_p = torch.tensor([1.0, 0.9, 1.0, 1.0] * (S // 4))
    seed = torch.arange(S, dtype=torch.int64) + 11
    stream = torch.arange(S, dtype=torch.int64) * 3
    c_dev = torch.arange(S, dtype=torch.int64) * 7
    c_ref = c_dev.clone()
    tok_d, n_d = verify(logits.to(cuda), drafts, temp, top_k, top_p, seed, stream, c_dev, q)
    tok_r, n_r = verify_ref(logits, drafts, temp, top_k, top_p, seed, stream, c_ref, q)
    assert torch.equal(n_d, n_r)
    assert torch.equal(c_dev, c_ref)
    for s in range(S):
        k = int(n_r[s]) + 1
        assert tok_d[s, :k].tolist() == tok_r[s, :k].tolist(), s


@pytest.mark.parametrize("k", [8, 6])
def test_moe_combine_rmsnorm_matches_reference(cuda, k):
    """Ordered combine of the top-k pair rows (+ shared expert) into the residual, then the next
    RMSNorm: top-8 (indices read once, the eight row loads issued together) and the generic
    loop; the residual equals the host's same-order f32 sum bit for bit."""
    torch.manual_seed(k)
    T, H = 37, 4096
    yp = torch.randn(T * k, H)
    pair_of = torch.randperm(T * k).view(T, k).to(torch.int32)
    shared = torch.randn(T, H)
    w = torch.rand(H) + 0.5
    x = torch.randn(T, H)
    xd, out = x.clone().to(cuda), torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
    ops.moe_combine_rmsnorm(xd, yp.to(cuda), pair_of.to(cuda), shared.to(cuda), w.to(cuda), out, 1e-6)
    xr, outr = x.clone(), torch.empty(T, H)
    ops.moe_combine_rmsnorm(xr, yp, pair_of, shared, w, outr, 1e-6)
    assert torch.equal(xd.cpu(), xr)
    assert _rel(out.float().cpu(), outr) < 1e-2
