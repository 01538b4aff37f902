"""Expert parallelism over NVLink on 2 GPUs: the fused dispatch/combine data plane gives
the same greedy tokens as the NCCL baseline data plane and as one GPU holding every expert.
Runs as two child processes (one per GPU); skipped with fewer than 2 GPUs."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import json, os, sys, torch
sys.path.insert(0, os.environ["ROOT"])
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner
from syntropy_b200.parallel.dist import init_distributed, shutdown
from syntropy_b200.parallel.ep import EPGroup
fused = os.environ["FUSED"] == "1"
spec_on = os.environ.get("SPEC") == "1"
ctx = init_distributed(timeout_s=60)
cfg = get_config(os.environ.get("MODEL", "small-qwen-moe"))
# MTP verify windows hold 2 rows per sequence
ep = EPGroup(ctx, cfg.n_experts, cfg.top_k, cfg.hidden, cap=8 if spec_on else 4, n_layers=cfg.n_layers, fused=fused)
if cfg.weight_quant == "fp8":  # the same synthetic weights the test's f32 reference uses
    from syntropy_b200.models.weights import synthetic_state_dict
    mw = prepare_weights(cfg, ctx.device, state_dict=synthetic_state_dict(cfg, seed=7), expert_range=ep.expert_range)
else:
    mw = prepare_weights(cfg, ctx.device, seed=7, expert_range=ep.expert_range)
runner = ModelRunner(mw, max_batch=8 if spec_on else 4, max_seq_len=256, ep=ep, use_graphs=fused)
spec = None
if spec_on:
    from syntropy_b200.runtime.spec import MTPDrafter, SpecConfig
    spec = SpecConfig(drafter=MTPDrafter(runner))
eng = LLMEngine(runner, dist_ctx=ctx, spec=spec)
g = torch.Generator().manual_seed(3)
prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (11, 30, 7, 19)]
outs = eng.generate(prompts[ctx.rank::ctx.world], SamplingParams(max_tokens=8))
st = ep.check_status()
runner.graphs.clear()
acc = eng.stats.get("spec_accepted", 0) / max(1, eng.stats.get("spec_drafted", 0)) if spec_on else None
print("RESULT " + json.dumps({"rank": ctx.rank, "outs": outs, "status": st, "accept": acc}), flush=True)
shutdown(ctx)
"""


def _run(fused: bool, model: str = "small-qwen-moe", spec: bool = False, port: int | None = None):
    port = port or (29611 if fused else 29612)
    procs = []
    for r in range(2):
        env = dict(os.environ, ROOT=ROOT, FUSED="1" if fused else "0", RANK=str(r), WORLD_SIZE="2",
                   LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                   MODEL=model, SPEC="1" if spec else "0")
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    res = {}
    for p in procs:
        out, _ = p.communicate(timeout=600)
        assert p.returncode == 0, out[-3000:]
        line = [x for x in out.splitlines() if x.startswith("RESULT ")][-1]
        d = json.loads(line[7:])
        res[d["rank"]] = d
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_fused_matches_baseline_and_single_gpu():
    from syntropy_b200.models.config import get_config
    from syntropy_b200.models.transformer import prepare_weights
    from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
    from syntropy_b200.runtime.runner import ModelRunner
    fused = _run(True)
    base = _run(False)
    same = 0
    for r in (0, 1):
        assert fused[r]["status"] == 0
        same += sum(a == b for a, b in zip(fused[r]["outs"], base[r]["outs"]))
    # fused sums the k expert rows per token; the baseline sums per-rank partials first:
    # the f32 association differs, so a near-tie argmax may flip on a random-weight model
    assert same >= 3
    cfg = get_config("small-qwen-moe")
    mw = prepare_weights(cfg, torch.device("cuda:0"), seed=7)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (11, 30, 7, 19)]
    single = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=256)).generate(prompts, SamplingParams(max_tokens=8))
    agree = sum(a == b for r in (0, 1) for a, b in zip(fused[r]["outs"], single[r::2]))
    assert agree >= 3  # different f32 summation association (per-rank partials) may flip a near-tie


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_fused_fp8_deepseek_with_mtp_follows_reference():
    """DeepSeek-style layers (MLA, block-scaled fp8 experts, a shared expert, group-limited
    routing) through the fused dispatch/combine, with and without MTP drafts verified in the
    same decode graphs: every emitted token is checked teacher-forced against the f32 reference
    forward over the fp8-rounded weights (the bound of the single-GPU fp8 engine test: e4m3
    activations flip near-ties of this random-weight model)."""
    from syntropy_b200.models import reference
    from syntropy_b200.models.config import get_config
    from syntropy_b200.models.weights import synthetic_state_dict
    from test_gpu_mla import _fp8_roundtrip_state
    plain = _run(True, "small-deepseek", spec=False, port=29613)
    spec = _run(True, "small-deepseek", spec=True, port=29614)
    for r in (0, 1):
        assert plain[r]["status"] == 0 and spec[r]["status"] == 0
        assert spec[r]["accept"] is not None
    cfg = get_config("small-deepseek")
    sdq = _fp8_roundtrip_state(synthetic_state_dict(cfg, seed=7))
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (11, 30, 7, 19)]
    for res in (plain, spec):
        agree = total = 0
        for r in (0, 1):
            for p, o in zip(prompts[r::2], res[r]["outs"]):
                logits = reference.forward(torch.tensor(p + o), sdq, cfg)
                ref_next = torch.argmax(logits[len(p) - 1:-1], -1).tolist()
                agree += sum(int(x == y) for x, y in zip(ref_next, o))
                total += len(o)
        assert agree / total >= 0.6, (agree, total, res)


TP_WORKER = r"""
import json, os, sys, torch
sys.path.insert(0, os.environ["ROOT"])
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.models.weights import synthetic_state_dict
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner
from syntropy_b200.parallel.dist import init_distributed, shutdown
from syntropy_b200.parallel.tp import TPGroup
fused = os.environ["FUSED"] == "1"
ctx = init_distributed(timeout_s=60)
cfg = get_config("small-llama")
sd = synthetic_state_dict(cfg, seed=9)
mw = prepare_weights(cfg, ctx.device, state_dict=sd, tp=(ctx.rank, ctx.world))
tp = TPGroup(ctx, cfg.hidden, cap=4, n_layers=cfg.n_layers, fused=fused)
runner = ModelRunner(mw, max_batch=4, max_seq_len=256, tp=tp, use_graphs=fused)
eng = LLMEngine(runner)
g = torch.Generator().manual_seed(3)
prompts = [torch.randint(0, cfg.vocab, (n,), generator=g).tolist() for n in (11, 30, 7)]
outs = eng.generate(prompts, SamplingParams(max_tokens=8))
st = tp.check_status()
runner.graphs.clear()
print("RESULT " + json.dumps({"rank": ctx.rank, "outs": outs, "status": st}), flush=True)
shutdown(ctx)
"""


def _run_tp(fused: bool):
    port = 29621 if fused else 29622
    procs = []
    for r in range(2):
        env = dict(os.environ, ROOT=ROOT, FUSED="1" if fused else "0", RANK=str(r), WORLD_SIZE="2",
                   LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", TP_WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    res = {}
    for p in procs:
        out, _ = p.communicate(timeout=600)
        assert p.returncode == 0, out[-3000:]
        d = json.loads([x for x in out.splitlines() if x.startswith("RESULT ")][-1][7:])
        res[d["rank"]] = d
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_fused_allreduce_ranks_agree_and_match_baseline():
    fused = _run_tp(True)
    base = _run_tp(False)
    assert fused[0]["status"] == 0 and fused[1]["status"] == 0
    # rank-order f32 reduction: both ranks hold identical residuals, so identical tokens
    assert fused[0]["outs"] == fused[1]["outs"]
    assert sum(a == b for a, b in zip(fused[0]["outs"], base[0]["outs"])) >= 2
