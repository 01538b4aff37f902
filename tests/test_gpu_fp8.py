"""Block-scaled fp8 kernels against plain f32 PyTorch references: the tiled weight layout
round trip, 1x128 activation quantisation, and the e4m3 x e4m3 GEMV (dense and grouped)
whose exact contract is  y = sum_b s_w s_x (q_w . q_x)  over 128-column blocks."""
import pytest
import torch

from syntropy_b200 import ops
from syntropy_b200._ext import ext
from syntropy_b200.formats.fp8 import FP8Weight, dequant_fp8_block, quantize_act_fp8

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _act_ref(xq, xs):
    T, K = xq.shape
    return xq.view(torch.float8_e4m3fn).float() * xs.repeat_interleave(128, 1)[:, :K]


def test_fp8_tiling_roundtrip_and_act_quant(cuda):
    torch.manual_seed(0)
    w = torch.randn(576, 1024, device=cuda) * 0.02
    W = FP8Weight.quantize(w)
    assert W.tiled is not None and W.tiled.numel() == 576 * 1024
    q, s = __import__("syntropy_b200.formats.fp8", fromlist=["x"]).quantize_fp8_block(w)
    assert torch.equal(W.rows().view(torch.uint8), q.view(torch.uint8))
    x = (torch.randn(7, 1024, device=cuda) * 3).to(torch.bfloat16)
    xq, xs = ext().f8_quant_act(x)
    rq, rs = quantize_act_fp8(x.float())
    assert torch.allclose(xs, rs, rtol=1e-6, atol=0)
    # multiplying by the reciprocal scale may round a boundary value the other way
    mism = (xq != rq.view(torch.uint8)).float().mean().item()
    assert mism < 1e-3, mism
    assert _rel(_act_ref(xq, xs), x.float()) < 0.04


@pytest.mark.parametrize("T,N,K,mode", [(1, 1024, 1024, "bf16"), (5, 576, 1024, "f32"), (16, 2048, 7168, "add"),
                                         (32, 1024, 512, "swiglu"), (3, 24576 // 8, 1536, "bf16"),
                                         (2, 576, 7168, "f32"), (16, 512, 18432, "swiglu")])
def test_fp8_gemv_dense(cuda, T, N, K, mode):
    torch.manual_seed(1)
    W = FP8Weight.quantize(torch.randn(N, K, device=cuda) * 0.02)
    wf = dequant_fp8_block(W.rows(), W.scale)
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    xq, xs = ext().f8_quant_act(x)
    ref = _act_ref(xq, xs) @ wf.t()
    if mode == "swiglu":
        out = torch.empty(T, N // 2, dtype=torch.bfloat16, device=cuda)
        ops.linear(x, W, out, ops.GEMV_SWIGLU)
        assert _rel(out, ops.swiglu_interleaved_ref(ref)) < 1e-2
    elif mode == "add":
        base = torch.randn(T, N, device=cuda)
        out = base.clone()
        ops.linear(x, W, out, ops.GEMV_ADD_F32)
        assert _rel(out - base, ref) < 1e-5
    elif mode == "f32":
        out = torch.empty(T, N, device=cuda)
        ops.linear(x, W, out, ops.GEMV_STORE)
        assert _rel(out, ref) < 1e-5
    else:
        out = torch.empty(T, N, dtype=torch.bfloat16, device=cuda)
        ops.linear(x, W, out, ops.GEMV_STORE)
        assert _rel(out, ref) < 5e-3


def test_fp8_gemv_grouped_scaled(cuda):
    torch.manual_seed(2)
    E, N, K, T = 6, 512, 1024, 9
    Ws = [FP8Weight.quantize(torch.randn(N, K, device=cuda) * 0.02) for _ in range(E)]
    qp = torch.tensor([w.tiled.data_ptr() for w in Ws], dtype=torch.int64, device=cuda)
    sp = torch.tensor([w.scale.data_ptr() for w in Ws], dtype=torch.int64, device=cuda)
    counts = [3, 0, 5, 1, 9, 2]
    off = [0]
    for c in counts:
        off.append(off[-1] + c)
    P = off[-1]
    tok_idx = torch.randint(0, T, (P,), dtype=torch.int32, device=cuda)
    route_w = torch.rand(P, device=cuda)
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    xq, xs = ext().f8_quant_act(x)
    out = torch.zeros(P, N, device=cuda)
    ext().f8_gemv(xq, xs, qp, sp, torch.tensor(off, dtype=torch.int32, device=cuda), tok_idx, route_w, out, N, K, 2, 2,
                  torch.empty(0, device=cuda))
    xa = _act_ref(xq, xs)
    ref = torch.zeros(P, N, device=cuda)
    for e in range(E):
        a, b = off[e], off[e + 1]
        if a < b:
            wf = dequant_fp8_block(Ws[e].rows(), Ws[e].scale)
            ref[a:b] = route_w[a:b, None] * (xa[tok_idx[a:b].long()] @ wf.t())
    assert _rel(out, ref) < 1e-5


@pytest.mark.parametrize("T,N,K", [(300, 576, 1024), (1024, 2048, 7168)])
def test_fp8_prefill_dequant_and_gemm(cuda, T, N, K):
    """Prefill rows over fp8 weights: the tiled dequant kernel equals the block-scale dequant of
    the row-major bytes exactly, and the prefill linear (dequant + tcgen05 bf16 GEMM) matches
    the f32 product with the dequantised weights."""
    torch.manual_seed(T)
    W = FP8Weight.quantize(torch.randn(N, K, device=cuda) * 0.02)
    wd = ext().f8_dequant_tiled(W.tiled, W.scale, N, K)
    ref_w = dequant_fp8_block(W.rows(), W.scale).to(torch.bfloat16)
    assert torch.equal(wd, ref_w)
    x = (torch.randn(T, K, device=cuda) * 0.5).to(torch.bfloat16)
    out = torch.empty(T, N, dtype=torch.float32, device=cuda)
    ops.linear(x, W, out, ops.GEMV_STORE)
    assert _rel(out, x.float() @ ref_w.float().t()) < 1e-4
