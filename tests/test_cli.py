"""The command line as a user runs it (`python -m syntropy_b200 ...`, CPU only): version,
resolved config with origins, placement plans (with the CPU share of the host tier on one
GPU), a constrained `run` on the tiny model, and the diagnostic bundle."""
import json
import os
import subprocess
import sys
import tarfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cli(*args, env=None):
    e = dict(os.environ, PYTHONPATH=ROOT, **(env or {}))
    r = subprocess.run([sys.executable, "-m", "syntropy_b200", *args], capture_output=True, text=True,
                       timeout=300, env=e, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_version_config_plan():
    assert json.loads(_cli("version"))["arch"] == "sm_100a"
    cfg = json.loads(_cli("-o", "tier.expert_cache_frac=0.6", "config", env={"SYN_SCHED_MAX_BATCH": "16"}))
    assert cfg["config"]["tier"]["expert_cache_frac"] == 0.6 and cfg["config"]["sched"]["max_batch"] == 16
    assert cfg["origin"]["sched.max_batch"] == "env SYN_SCHED_MAX_BATCH"
    plan = json.loads(_cli("-o", "model.name=qwen3-235b-a22b", "plan", "--gpus", "1", "--expert-cache-frac", "0.6"))
    assert plan["mode"] == "local" and plan["cpu_expert_share"] > 0.5
    plan8 = json.loads(_cli("-o", "model.name=qwen3-235b-a22b", "plan", "--gpus", "8"))
    assert plan8["cpu_expert_share"] == 0


def test_run_with_choice_constraint_and_bundle(tmp_path):
    out = json.loads(_cli("-o", "model.name=tiny-llama", "-o", "model.max_seq_len=64", "-o", "sched.max_batch=2",
                          "run", "--prompt", "pick", "--max-tokens", "8", "--choices", "left|right", "--device", "cpu"))
    assert out["text"] in ("left", "right")
    path = _cli("bundle", "--out", str(tmp_path / "b.tar.gz"), "--crash-dir", str(tmp_path / "none")).strip()
    with tarfile.open(path) as t:
        assert "config.json" in t.getnames()
