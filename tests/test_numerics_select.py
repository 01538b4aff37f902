"""Numerics contract: tolerance classes, the accumulation-precision detector, and provider
selection (certificate against the f32 reference, then timing with a 3% margin for the
default, cached and persisted decisions)."""
import torch

from syntropy_b200.ops.numerics import TOLERANCES, Candidate, Selector, accumulation_class, within


def test_accumulation_detector():
    assert accumulation_class(lambda x, w: x.float() @ w.float().t()) == "f32"

    def bf16_acc(x, w):  # adds the products one at a time in bf16
        acc = torch.zeros(1, dtype=torch.bfloat16)
        for a, b in zip(x[0], w[0]):
            acc = (acc + a * b).to(torch.bfloat16)
        return acc
    assert accumulation_class(bf16_acc, n=512) == "reduced"


def _const(out):
    return lambda *a: out


def test_selector_certifies_times_and_prefers_the_default():
    want = torch.randn(8, 8)
    times = {"default": 10.0, "slightly": 9.8, "fast": 8.0, "wrong": 1.0}
    sel = Selector(timer=lambda name, fn: times[name])
    cands = [Candidate("default", _const(want), "bf16_f32acc"), Candidate("slightly", _const(want), "bf16_f32acc"),
             Candidate("wrong", _const(want + 1.0), "bf16_f32acc")]
    assert sel.choose("op", (8, 8), cands, (), lambda: want) == "default"  # 2% faster is not enough
    log = {r["candidate"]: r["certified"] for r in sel.log if "candidate" in r}
    assert log["wrong"] is False and log["slightly"] is True  # the fastest is wrong: never chosen
    cands.append(Candidate("fast", _const(want), "bf16_f32acc"))
    assert sel.choose("op", (16, 8), cands, (), lambda: want) == "fast"
    assert sel.choose("op", (8, 8), cands, (), lambda: want) == "default"  # cached


def test_selector_save_load(tmp_path):
    sel = Selector(decisions={"op:1x2": "fast"})
    sel.save(str(tmp_path / "sel.json"))
    s2 = Selector()
    s2.load(str(tmp_path / "sel.json"))
    assert s2.decisions == {"op:1x2": "fast"}


def test_tolerance_classes():
    a = torch.randn(100)
    assert within("f32", a * (1 + 1e-7), a) and not within("f32", a * 1.01, a)
    assert TOLERANCES["bf16_out"] > TOLERANCES["bf16_f32acc"]
