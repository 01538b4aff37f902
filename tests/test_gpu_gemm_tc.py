"""tcgen05 prefill GEMM (4-bit weights, grouped) against an f32 PyTorch matmul of the
dequantised weights."""
import pytest
import torch

from syntropy_b200 import ops
from syntropy_b200._ext import ext
from syntropy_b200.formats.q4 import Q4Weight

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 256, 256), (300, 128, 512), (1000, 512, 1024)])
def test_tc_gemm_dense(cuda, M, N, K):
    torch.manual_seed(0)
    w = torch.randn(N, K, device=cuda) * 0.02
    q = Q4Weight.quantize(w)
    wd = q.dequant().float()
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.zeros(M, N, dtype=torch.float32, device=cuda)
    ptrs = (torch.tensor([q.qw.data_ptr()], device=cuda), torch.tensor([q.sm.data_ptr()], device=cuda))
    off = torch.tensor([0, M], dtype=torch.int32, device=cuda)
    e = torch.empty(0, dtype=torch.int32, device=cuda)
    ext().tc_gemm_q4(x, ptrs[0], ptrs[1], off, N, K, 5, torch.empty(0, device=cuda), out, status, (M + 127) // 128 + 1,
                     e, e, 0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = x.float() @ wd.t()
    # wd is the format's dequantised bf16 value: the kernel must produce exactly these
    # weights, so only the f32 summation order differs
    assert _rel(out, ref) < 2e-5
    ob = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda)
    ext().tc_gemm_q4(x, ptrs[0], ptrs[1], off, N, K, 0, torch.empty(0, device=cuda), ob, status, (M + 127) // 128 + 1,
                     q.qw, q.sm, 0)
    assert _rel(ob, ref) < 5e-3
    # TMA-streamed weights give the same result as the bulk-copy path
    ot = torch.zeros(M, N, dtype=torch.float32, device=cuda)
    ext().tc_gemm_q4(x, ptrs[0], ptrs[1], off, N, K, 5, torch.empty(0, device=cuda), ot, status, (M + 127) // 128 + 1,
                     q.qw, q.sm, 0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and torch.equal(ot, out)


def test_tc_gemm_grouped_swiglu_scaled(cuda):
    torch.manual_seed(1)
    G, f, H = 5, 128, 256
    counts = [0, 130, 7, 256, 1]
    g = torch.randn(G, f, H, device=cuda) * 0.02
    u = torch.randn(G, f, H, device=cuda) * 0.02
    qs = [Q4Weight.quantize(ops.interleave_gate_up(g[e], u[e])) for e in range(G)]
    M = sum(counts)
    off = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32, device=cuda)
    x = torch.randn(M, H, device=cuda).to(torch.bfloat16)
    qp = torch.tensor([q.qw.data_ptr() for q in qs], device=cuda)
    sp = torch.tensor([q.sm.data_ptr() for q in qs], device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    mid = torch.zeros(M, f, dtype=torch.bfloat16, device=cuda)
    e = torch.empty(0, dtype=torch.int32, device=cuda)
    ext().tc_gemm_q4(x, qp, sp, off, 2 * f, H, 1, torch.empty(0, device=cuda), mid, status, M // 128 + G + 1, e, e, 0)
    rw = torch.rand(M, device=cuda)
    y = torch.zeros(M, 2 * f, dtype=torch.float32, device=cuda)
    bq = torch.stack([q.qw for q in qs])
    bs = torch.stack([q.sm for q in qs])
    qp2 = torch.tensor([bq[i].data_ptr() for i in range(G)], device=cuda)
    sp2 = torch.tensor([bs[i].data_ptr() for i in range(G)], device=cuda)
    ext().tc_gemm_q4(x, qp2, sp2, off, 2 * f, H, 2, rw, y, status, M // 128 + G + 1, bq, bs, 0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    offs = off.tolist()
    for e in range(G):
        a, b = offs[e], offs[e + 1]
        if a == b:
            continue
        ref = x[a:b].float() @ qs[e].dequant().float().t()
        assert _rel(mid[a:b], ops.swiglu_interleaved_ref(ref)) < 1e-2
        assert _rel(y[a:b], rw[a:b, None] * ref) < 2e-3
