"""Allocation-free C entry point of the dense decode GEMV against the torch op and an f32
reference.  Collected last on purpose: it must pass both alone and after every other test."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from syntropy_b200._ext import ext
    lib = ctypes.CDLL(ext().__file__)
    fn = lib.syn_q4_gemv_dense_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return fn


def _call(fn, x, q, out, mode):
    err = ctypes.create_string_buffer(256)
    rc = fn(x.data_ptr(), x.shape[0], x.stride(0), q.qw.data_ptr(), q.sm.data_ptr(), out.data_ptr(), q.N, q.K, mode,
            torch.cuda.current_stream().cuda_stream, err, 256)
    return rc, err.value.decode()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,N,K,mode", [(32, 9216, 4096, 0), (16, 4096, 8192, 5), (24, 3072, 4096, 1),
                                         (9, 1024, 1536, 3), (4, 512, 512, 0), (64, 2048, 4096, 5)])
def test_noalloc_matches_torch_op(cuda, T, N, K, mode):
    from syntropy_b200._ext import ext
    from syntropy_b200.formats.q4 import Q4Weight, dequant_rows_ref
    fn = _lib()
    torch.manual_seed(11)
    q = Q4Weight.quantize(torch.randn(N, K, device=cuda) * 0.02)
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    ref = x.float() @ dequant_rows_ref(q.to_rows().cpu(), N, K).to(cuda).t()
    ncols = N // 2 if mode == 1 else N
    dt = torch.bfloat16 if mode in (0, 1) else torch.float32
    # the existing torch entry point, with its own workspace
    ptrs = (torch.tensor([q.qw.data_ptr()], dtype=torch.int64, device=cuda),
            torch.tensor([q.sm.data_ptr()], dtype=torch.int64, device=cuda))
    off = torch.tensor([0, T], dtype=torch.int32, device=cuda)
    ws = torch.empty(max(1, ext().q4_gemv_dense_ws(N, K, T)), dtype=torch.float32, device=cuda)
    ctr = torch.zeros(N // 64, dtype=torch.int32, device=cuda)
    base = torch.randn(T, ncols, device=cuda).to(dt) if mode == 3 else torch.zeros(T, ncols, dtype=dt, device=cuda)
    want = base.clone()
    ext().q4_gemv_dense(x, ptrs[0], ptrs[1], off, want, N, K, mode, ws, ctr)
    for _ in range(2):  # two calls in a row: the shared scratch must not carry state over
        got = base.clone()
        rc, msg = _call(fn, x, q, got, mode)
        assert rc == 0, msg
        torch.cuda.synchronize()
        if mode == 3:
            assert _rel(got - base, want - base) < 1e-5
            assert _rel(got - base, ref) < 1e-4
        elif mode == 5:
            assert _rel(got, want) < 1e-5
            assert _rel(got, ref) < 1e-4
        elif mode == 1:
            assert _rel(got, want) < 1e-2
        else:
            assert _rel(got, want) < 5e-3
            assert _rel(got, ref) < 5e-3


def test_noalloc_rejects_sizes_beyond_scratch(cuda):
    from syntropy_b200.formats.q4 import Q4Weight
    fn = _lib()
    N, K = 151936, 4096  # a vocabulary-sized head: its split-K workspace is larger than the fixed scratch
    q = Q4Weight(N, K, torch.zeros(1, dtype=torch.int32, device=cuda), torch.zeros(1, dtype=torch.float16, device=cuda))
    x = torch.zeros(32, K, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(1, dtype=torch.bfloat16, device=cuda)
    rc, msg = _call(fn, x, q, out, 0)
    assert rc == -1 and "scratch" in msg
    x2 = torch.zeros(65, 64, dtype=torch.bfloat16, device=cuda)
    rc, msg = _call(fn, x2, q, out, 0)
    assert rc == -1 and "rows" in msg
