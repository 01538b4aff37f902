"""4-bit decode GEMM on tcgen05 (csrc/cuda/gemm_q4_dec.cu: dequantised weights as the M = 128
operand, 16-64 token rows as N, K split over a thread-block cluster) against a plain f32
PyTorch reference over the dequantised weights, for every epilogue, and the linear dispatch
that routes 16-64 rows there."""
import pytest
import torch

from syntropy_b200 import ops
from syntropy_b200._ext import ext
from syntropy_b200.formats.q4 import Q4Weight
from syntropy_b200.ops.core import gemm_status, swiglu_interleaved_ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,N,K", [(16, 1024, 1024), (32, 8192, 8192), (33, 10240, 4096), (64, 1280, 8192),
                                   (1, 256, 512), (48, 8192, 28672)])
@pytest.mark.parametrize("mode", [0, 1, 3, 5])
def test_q4_gemm_dec_modes(cuda, T, N, K, mode):
    torch.manual_seed(T + N + mode)
    W = Q4Weight.quantize(torch.randn(N, K, device=cuda) * 0.02)
    wd = W.dequant().float()
    x = (torch.randn(T, K, device=cuda) * 0.5).to(torch.bfloat16)
    ref = x.float() @ wd.t()
    st = gemm_status(cuda)
    st.zero_()
    if mode == 0:
        out, want = torch.empty(T, N, dtype=torch.bfloat16, device=cuda), ref
    elif mode == 1:
        out, want = torch.empty(T, N // 2, dtype=torch.bfloat16, device=cuda), swiglu_interleaved_ref(ref)
    elif mode == 3:
        out = torch.randn(T, N, device=cuda)
        want = out.clone() + ref
    else:
        out, want = torch.empty(T, N, dtype=torch.float32, device=cuda), ref
    ext().q4_gemm_dec(x, W.qw, W.sm, N, K, mode, out, st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    # the dequantised weight is rounded to bf16 once (d*q+m in f32): the bf16 class for f32 outputs
    tol = 1e-2 if mode in (0, 1) else 5e-3
    assert _rel(out, want) < tol, (T, N, K, mode, _rel(out, want))


def test_linear_routes_16_to_64_rows_to_tcgen05(cuda):
    """ops.linear over 4-bit weights at 32 rows (tcgen05) against the GEMV path (SYN_Q4_TC_MIN
    above 64) and the f32 reference."""
    from syntropy_b200.ops import core
    torch.manual_seed(1)
    W = Q4Weight.quantize(torch.randn(4096, 4096, device=cuda) * 0.02)
    x = (torch.randn(32, 4096, device=cuda) * 0.5).to(torch.bfloat16)
    a = torch.zeros(32, 4096, device=cuda)
    b = torch.zeros(32, 4096, device=cuda)
    ops.linear(x, W, a, ops.GEMV_ADD_F32)
    saved = core._Q4_TC[0]
    core._Q4_TC[0] = 1 << 30
    try:
        ops.linear(x, W, b, ops.GEMV_ADD_F32)
    finally:
        core._Q4_TC[0] = saved
    # the GEMV folds scale and min in f32; the tcgen05 path rounds each dequantised weight to
    # bf16 once (as the prefill GEMM does): both within the bf16-weight bound of the reference
    ref = x.float() @ W.dequant().float().t()
    assert _rel(a, ref) < 5e-3 and _rel(b, ref) < 5e-3
    assert _rel(a, b) < 5e-3
