"""End-to-end engine on the GPU against the f32 reference forward (same q4-dequantised
weights), for the Qwen3-MoE and Llama families."""
import pytest
import torch

from syntropy_b200.formats.q4 import dequant_rows_ref
from syntropy_b200._ext import ext
from syntropy_b200.models import reference
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner

pytestmark = pytest.mark.gpu


def _q4_roundtrip_state(sd):
    """Replace every linear weight by its q4-dequantised value (what the GPU computes with)."""
    out = {}
    for n, t in sd.items():
        if t.dim() >= 2 and not n.endswith("embed") and not n.endswith("router"):
            flat = t.reshape(-1, t.shape[-1])
            rows = ext().q4_quantize_rows_cpu(flat.float().contiguous())
            out[n] = dequant_rows_ref(rows, flat.shape[0], flat.shape[1]).reshape(t.shape)
        elif n.endswith("embed") or n.endswith("router"):
            out[n] = t.to(torch.bfloat16).float()
        else:
            out[n] = t
    return out


@pytest.mark.parametrize("name", ["small-qwen-moe", "small-llama"])
def test_engine_logits_match_reference(cuda, name):
    cfg = get_config(name)
    sd = synthetic_state_dict(cfg, seed=3)
    sdq = _q4_roundtrip_state(sd)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (40, 9, 77)]
    mw = prepare_weights(cfg, cuda, state_dict=sd)
    runner = ModelRunner(mw, max_batch=8, max_seq_len=256)
    eng = LLMEngine(runner)
    outs = eng.generate(prompts, SamplingParams(max_tokens=6))
    # teacher-forced check: reference logits on prompt + engine outputs, top-1 agreement
    agree, total = 0, 0
    for p, o in zip(prompts, outs):
        toks = torch.tensor(p + o)
        logits = reference.forward(toks, sdq, cfg)
        ref_next = torch.argmax(logits[len(p) - 1:-1], -1).tolist()
        agree += sum(int(a == b) for a, b in zip(ref_next, o))
        total += len(o)
    assert agree / total >= 0.85, (agree, total)


def test_cuda_graph_decode_equals_eager(cuda):
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, cuda, seed=5)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (12, 30, 7, 64, 3)]
    a = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=True)).generate(
        prompts, SamplingParams(max_tokens=10))
    b = LLMEngine(ModelRunner(mw, max_batch=8, max_seq_len=256, use_graphs=False)).generate(
        prompts, SamplingParams(max_tokens=10))
    assert a == b
