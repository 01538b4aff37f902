"""MLA decode kernel (absorbed, latent 512 + rope 64, paged latent cache) against a plain
f32 PyTorch reference, and the fp8 DeepSeek-shaped model on the GPU engine: CUDA-graph
decode equals eager decode, greedy tokens follow the f32 reference forward."""
import math

import pytest
import torch

from syntropy_b200 import ops
from syntropy_b200.models import reference
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,ctx,pps", [(128, [1, 33, 700], 8), (16, [300, 5], 3), (32, [2048], 16)])
def test_mla_decode_kernel(cuda, H, ctx, pps):
    torch.manual_seed(3)
    B = len(ctx)
    need = [(c + 15) // 16 for c in ctx]
    nb = sum(need) + 2
    perm = (torch.randperm(nb - 1) + 1).tolist()
    width = max(need) + 3
    bt = torch.zeros(B, width, dtype=torch.int32)
    o = 0
    for r, k in enumerate(need):
        bt[r, :k] = torch.tensor(perm[o:o + k], dtype=torch.int32)
        o += k
    cache = torch.randn(nb, 16, 576, device=cuda).to(torch.bfloat16)
    q = torch.randn(B, H, 576, device=cuda).to(torch.bfloat16)
    scale = 1 / math.sqrt(192)
    ns = -(-width // pps)
    po = torch.empty(B * H * ns * 512, device=cuda)
    pml = torch.empty(B * H * ns * 2, device=cuda)
    out = torch.empty(B, H, 512, device=cuda)
    ops.mla_decode(q, cache, bt.to(cuda), torch.tensor(ctx, dtype=torch.int32, device=cuda), out, scale, po, pml, pps)
    flat = cache.view(-1, 576).float()
    for r in range(B):
        pos = torch.arange(ctx[r], device=cuda)
        rows = flat[bt[r].to(cuda)[pos // 16].long() * 16 + pos % 16]
        s = (q[r].float() @ rows.t()) * scale
        ref = torch.softmax(s, -1) @ rows[:, :512]
        err = ((out[r] - ref).norm() / ref.norm()).item()
        assert err < 1e-2, (r, err)


def _fp8_roundtrip_state(sd):
    """The weights as the engine stores them: every fp8 matrix quantised and dequantised the
    way prepare_weights builds it (gate/up interleaved in 8-row chunks before quantising)."""
    from syntropy_b200.formats.fp8 import FP8Weight

    def rt(t):
        return FP8Weight.quantize(t.float()).dequant(torch.float32)

    def rt_pair(g, u):
        f, H = g.shape
        w = rt(ops.interleave_gate_up(g.float(), u.float())).view(f // 8, 2, 8, H)
        return w[:, 0].reshape(f, H), w[:, 1].reshape(f, H)

    out = dict(sd)
    for n, t in sd.items():
        leaf = n.split(".")[-1]
        if n.startswith("mtp."):
            continue
        if n.endswith("experts.gate"):
            up = sd[n[:-4] + "up"]
            pairs = [rt_pair(t[e], up[e]) for e in range(t.shape[0])]
            out[n] = torch.stack([p[0] for p in pairs])
            out[n[:-4] + "up"] = torch.stack([p[1] for p in pairs])
        elif n.endswith("experts.down"):
            out[n] = torch.stack([rt(t[e]) for e in range(t.shape[0])])
        elif leaf in ("q_a", "q_b", "kv_a", "o_proj", "down") or n == "lm_head":
            if t.shape[0] % 16 == 0 and t.shape[1] % 128 == 0:
                out[n] = rt(t)
        elif leaf == "gate" and "experts" not in n:  # dense FFN and shared expert
            out[n], out[n[:-4] + "up"] = rt_pair(t, sd[n[:-4] + "up"])
    return out


def test_deepseek_fp8_engine(cuda):
    cfg = get_config("small-deepseek")
    sd = synthetic_state_dict(cfg, seed=7)
    mw = prepare_weights(cfg, cuda, state_dict=sd)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (30, 7, 50)]
    sp = SamplingParams(max_tokens=6)
    a = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, use_graphs=True)).generate(prompts, sp)
    b = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128, use_graphs=False)).generate(prompts, sp)
    assert a == b
    sdq = _fp8_roundtrip_state(sd)
    agree = total = 0
    for p, o in zip(prompts, a):
        toks = torch.tensor(p + o)
        logits = reference.forward(toks, sdq, cfg)
        ref_next = torch.argmax(logits[len(p) - 1:-1], -1).tolist()
        agree += sum(int(x == y) for x, y in zip(ref_next, o))
        total += len(o)
    assert agree / total >= 0.6, (agree, total)


def test_deepseek_fp8_mtp_spec(cuda):
    """MTP drafting + batched verification on the GPU: greedy tokens follow plain greedy
    decoding (the verify windows run the same model), and acceptance is reported."""
    from syntropy_b200.runtime.spec import MTPDrafter, SpecConfig
    cfg = get_config("small-deepseek")
    mw = prepare_weights(cfg, cuda, seed=9)
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (20, 41)]
    sp = SamplingParams(max_tokens=8)
    want = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate(prompts, sp)
    runner = ModelRunner(mw, max_batch=4, max_seq_len=128)
    eng = LLMEngine(runner, spec=SpecConfig(drafter=MTPDrafter(runner)))
    got = eng.generate(prompts, sp)
    same = sum(int(a == b) for x, y in zip(got, want) for a, b in zip(x, y))
    assert same / sum(len(x) for x in want) >= 0.75, (got, want)
    assert eng.stats["spec_drafted"] > 0 and 0.0 <= eng.acceptance_rate <= 1.0


@pytest.mark.parametrize("T", [1, 5, 19])
def test_mla_decode_projection_kernels(cuda, T):
    """mla_kv_write / mla_q_absorb / mla_o_absorb against the f32 tensor path they replace
    (mla_qkv's latent row and absorbed query, the W_uv einsum), on DeepSeek-V3 head shapes."""
    from syntropy_b200._ext import ext
    from syntropy_b200.models.mla import mla_qkv, mla_qkv_decode
    cfg = get_config("small-deepseek")
    mw = prepare_weights(cfg, cuda, seed=21)
    m = mw.layers[0].mla
    H = cfg.n_heads
    g = torch.Generator().manual_seed(T)
    h = torch.randn(T, cfg.hidden, generator=g).to(cuda, torch.bfloat16)
    pos = torch.randint(0, 100, (T,), generator=g).int().to(cuda)
    slot = torch.randperm(64, generator=g)[:T].long().to(cuda) + 16
    slot[0] = -1  # a padding row writes the null page
    cache = torch.zeros(8, 16, 576, dtype=torch.bfloat16, device=cuda)
    qcat = torch.empty(T, H, 576, dtype=torch.bfloat16, device=cuda)
    mla_qkv_decode(cfg, m, h, pos, slot, mw.rope_cos, mw.rope_sin, cache, qcat)
    q_lat, q_pe, lat = mla_qkv(cfg, m, h, pos, mw.rope_cos, mw.rope_sin)
    want_q = torch.cat([q_lat, q_pe], -1)
    assert ((qcat.float() - want_q).norm() / want_q.norm()).item() < 1e-2
    rows = cache.view(-1, 576)[torch.where(slot >= 0, slot, torch.zeros_like(slot))]
    assert ((rows.float() - lat).norm() / lat.norm()).item() < 1e-2
    o_lat = torch.randn(T, H, 512, generator=g).to(cuda)
    out = torch.empty(T, H * 128, dtype=torch.bfloat16, device=cuda)
    ext().mla_o_absorb(o_lat, m["w_uv"], out)
    want_o = torch.einsum("thc,hvc->thv", o_lat, m["w_uv"].float()).reshape(T, -1)
    assert ((out.float() - want_o).norm() / want_o.norm()).item() < 1e-2
