"""bf16 GEMM on tcgen05 (csrc/cuda/gemm_bf16_tc.cu) against a plain f32 PyTorch reference of
the same op: both orientations (decode below 128 rows with split-K, prefill from 128), every
epilogue, partial weight tiles (N % 128 != 0), a strided activation view, and the engine's
bf16 model path (greedy tokens against the f32 reference forward)."""
import pytest
import torch

from syntropy_b200 import ops
from syntropy_b200._ext import ext
from syntropy_b200.ops.core import _bf16_workspace, gemm_status, swiglu_interleaved_ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,N,K", [(1, 768, 4096), (7, 4096, 512), (32, 3584, 4096), (64, 4096, 1792),
                                   (100, 1024, 1024), (128, 768, 4096), (300, 4096, 1024), (1000, 2048, 512),
                                   (64, 16032, 4096), (5, 160, 256), (200, 160, 256)])
@pytest.mark.parametrize("mode", [0, 1, 3, 5])
def test_gemm_bf16_modes(cuda, T, N, K, mode):
    if mode == 1 and N % 16:
        pytest.skip("SwiGLU needs whole 16-row gate/up chunks")
    torch.manual_seed(T * 7 + N + mode)
    x = (torch.randn(T, K, device=cuda) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) * 0.02).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    ws, ctr = _bf16_workspace(cuda, N, K, T)
    st = gemm_status(cuda)
    if mode == 0:
        out = torch.empty(T, N, dtype=torch.bfloat16, device=cuda)
        want = ref
    elif mode == 1:
        out = torch.empty(T, N // 2, dtype=torch.bfloat16, device=cuda)
        want = swiglu_interleaved_ref(ref)
    elif mode == 3:
        out = torch.randn(T, N, device=cuda)
        want = out.clone() + ref
    else:
        out = torch.empty(T, N, dtype=torch.float32, device=cuda)
        want = ref
    ext().gemm_bf16(x, w, out, mode, ws, ctr, st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert int(ctr.abs().sum()) == 0, "split-K counters must be left at zero"
    tol = 1e-2 if mode in (0, 1) else 1e-4
    assert _rel(out, want) < tol, (T, N, K, mode, _rel(out, want))


def test_gemm_bf16_strided_rows_and_repeat(cuda):
    """x as a column slice of a wider buffer (row stride > K), two launches in a row (split-K
    counters and workspace reused)."""
    torch.manual_seed(3)
    buf = (torch.randn(48, 3 * 1024, device=cuda)).to(torch.bfloat16)
    x = buf[:, 1024:2048]
    w = (torch.randn(2048, 1024, device=cuda) * 0.02).to(torch.bfloat16)
    out = torch.empty(48, 2048, dtype=torch.float32, device=cuda)
    for _ in range(2):
        ops.linear(x, w, out, ops.GEMV_STORE)
    torch.cuda.synchronize()
    assert _rel(out, x.float() @ w.float().t()) < 1e-4


def test_bf16_model_matches_reference(cuda):
    """A small bf16 Llama-style model (every projection and the LM head on the tcgen05 GEMM):
    prefill logits of the last prompt token against the f32 reference forward over the same
    bf16-rounded weights, and a greedy decode through the engine runs to completion."""
    from syntropy_b200.models import reference
    from syntropy_b200.models.config import get_config
    from syntropy_b200.models.transformer import prepare_weights
    from syntropy_b200.models.weights import synthetic_state_dict
    from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
    from syntropy_b200.runtime.runner import ModelRunner
    cfg = get_config("small-llama").replace(weight_quant="bf16")
    sd = {k: v.to(torch.bfloat16).float() for k, v in synthetic_state_dict(cfg, seed=4).items()}
    mw = prepare_weights(cfg, cuda, state_dict=sd)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, cfg.vocab, (140,), generator=g).tolist()
    runner = ModelRunner(mw, max_batch=4, max_seq_len=256)
    blocks = list(range(1, 1 + (len(prompt) + 15) // 16))
    slots = torch.tensor([blocks[p // 16] * 16 + p % 16 for p in range(len(prompt))])
    got = runner.prefill(torch.tensor(prompt), torch.arange(len(prompt)), slots, [0, len(prompt)],
                         block_lists=[blocks])[0].float().cpu()
    want = reference.forward(torch.tensor(prompt), sd, cfg)[-1].float()
    assert _rel(got, want) < 5e-2
    assert int(got.argmax()) == int(want.argmax())
    out = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=256)).generate([prompt[:9], prompt[:33]],
                                                                           SamplingParams(max_tokens=6))
    assert all(len(o) == 6 for o in out)


def test_bf16_gemm_accumulates_in_f32_and_is_selectable(cuda):
    """The accumulation detector sees f32 accumulation in the tcgen05 GEMM; the selector certifies
    both providers of a decode shape against the f32 reference and picks one."""
    from syntropy_b200.ops import core
    from syntropy_b200.ops.numerics import Selector, accumulation_class

    def dot(x, w):
        o = torch.empty(1, 128, dtype=torch.float32, device=cuda)
        wp = torch.zeros(128, x.shape[1], dtype=torch.bfloat16, device=cuda)
        wp[0] = w[0]
        ws, ctr = _bf16_workspace(cuda, 128, x.shape[1], 1)
        ext().gemm_bf16(x, wp, o, 5, ws, ctr, gemm_status(cuda))
        return o[:, :1]
    assert accumulation_class(dot, device=cuda) == "f32"
    saved, core._BF16_TC[0], core.SELECTOR = core._BF16_TC[0], "auto", Selector()
    try:
        x = (torch.randn(64, 4096, device=cuda) * 0.5).to(torch.bfloat16)
        w = (torch.randn(1024, 4096, device=cuda) * 0.02).to(torch.bfloat16)
        out = torch.empty(64, 1024, dtype=torch.bfloat16, device=cuda)
        ops.linear(x, w, out, ops.GEMV_STORE)
        assert _rel(out, x.float() @ w.float().t()) < 1e-2
        certs = [r for r in core.SELECTOR.log if "certified" in r]
        assert {r["candidate"] for r in certs} == {"tcgen05", "library"} and all(r["certified"] for r in certs)
        assert list(core.SELECTOR.decisions.values())[0] in ("tcgen05", "library")
    finally:
        core._BF16_TC[0], core.SELECTOR = saved, None
