"""Parity harness: the engine against the naive f32 reference forward, teacher-forced.

The engine serves one sequence whose sampled token is replaced by the reference token before
every step (teacher forcing), so both see the same context at every position; the engine's
logits of each step (prefill for the first position, graph-replayed decode steps after it)
are compared with the reference logits of that position:

* top-1 agreement: share of positions where both argmaxes agree;
* KL(reference || engine) per position (f32 softmax), mean and max;
* max |logit difference| relative to the reference's logit spread.

`fidelity(...)` returns the report and `gate(...)` checks it against class ceilings
(reference RFC-0042 §5-§6 and RFC-0060: teacher-forced top-1 agreement + KL over a corpus vs
the F32 reference; crates/core/src/fidelity.rs).

    python -m syntropy_b200.bench.parity --model small-llama --tokens 64 [--device cuda:0]
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F

# ceilings by weight class: (min top-1 agreement, max mean KL)
CEILINGS = {"fp32": (1.0, 1e-6), "bf16": (0.97, 1e-3), "fp8": (0.93, 1e-2), "q4": (0.85, 5e-2)}


def engine_logits(engine, tokens: list[int]) -> torch.Tensor:
    """[T-1, V] logits of positions 0..T-2 (each predicting the next token), teacher-forced."""
    from ..runtime.engine import SamplingParams
    T = len(tokens)
    sid = engine.add_request(tokens[:1], SamplingParams(max_tokens=T))
    s = next(x for x in engine.waiting if x.seq_id == sid)
    out = []
    r = engine.runner
    # prefill of the first token: its logits come back from the runner
    orig = r.prefill

    def capture(*a, **k):
        lg = orig(*a, **k)
        out.append(lg[-1].detach().float().cpu().clone())
        return lg
    r.prefill = capture
    try:
        engine.step()
    finally:
        r.prefill = orig
    for t in range(1, T - 1):
        s.output[-1] = tokens[t]  # teacher forcing: the reference token is the next input
        engine.step()
        out.append(r.buf["logits"][0].detach().float().cpu().clone())
    engine.abort(sid)
    return torch.stack(out)


def fidelity(eng_logits: torch.Tensor, ref_logits: torch.Tensor) -> dict:
    n = min(len(eng_logits), len(ref_logits))
    a, b = eng_logits[:n].float(), ref_logits[:n].float()
    agree = (a.argmax(-1) == b.argmax(-1)).float().mean().item()
    kl = F.kl_div(F.log_softmax(a, -1), F.log_softmax(b, -1), log_target=True, reduction="none").sum(-1)
    spread = (b.amax(-1) - b.amin(-1)).clamp_min(1e-9)
    rel = ((a - b).abs().amax(-1) / spread).max().item()
    return {"positions": n, "top1_agreement": round(agree, 4), "kl_mean": float(kl.mean()), "kl_max": float(kl.max()),
            "max_rel_logit_err": rel}


def gate(report: dict, weight_class: str) -> bool:
    top1, kl = CEILINGS[weight_class]
    return report["top1_agreement"] >= top1 and report["kl_mean"] <= kl


def run(model: str, n_tokens: int, device: str = "cpu", seed: int = 0, use_graphs: bool = True) -> dict:
    from ..models import reference
    from ..models.config import get_config
    from ..models.transformer import prepare_weights
    from ..models.weights import synthetic_state_dict
    from ..runtime.engine import LLMEngine
    from ..runtime.runner import ModelRunner
    cfg = get_config(model)
    sd = synthetic_state_dict(cfg, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    tokens = torch.randint(3, cfg.vocab, (n_tokens,), generator=g).tolist()
    ref = reference.forward(torch.tensor(tokens), sd, cfg)[:-1]
    dev = torch.device(device)
    mw = prepare_weights(cfg, dev, state_dict=sd, max_pos=n_tokens + 16)
    eng = LLMEngine(ModelRunner(mw, max_batch=1, max_seq_len=n_tokens + 8, use_graphs=use_graphs))
    rep = fidelity(engine_logits(eng, tokens), ref)
    wc = cfg.weight_quant if dev.type == "cuda" else "fp32"
    rep.update({"model": model, "weights": wc, "device": device, "gate": gate(rep, wc)})
    return rep


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--tokens", type=int, default=48)
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    print(json.dumps(run(a.model, a.tokens, a.device, a.seed)))


if __name__ == "__main__":
    main()
