"""Diagnostics on CPU: credential redaction, crash records from an uncaught exception in a
child process, the bundle's contents, and repeat suppression in the logging pipeline."""
import json
import logging
import os
import subprocess
import sys
import tarfile

from syntropy_b200.config.schema import load_config
from syntropy_b200.daemon.bundle import REDACTED, make_bundle, redact
from syntropy_b200.obs.log import RepeatSuppressor

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_redaction():
    r = redact({"api_key": "abc", "nested": {"hf_token": "x", "n": 3},
                "url": "https://user:pw@host/x", "hdr": "Authorization: Bearer sk-123", "list": [{"password": 1}]})
    assert r["api_key"] == REDACTED and r["nested"]["hf_token"] == REDACTED and r["nested"]["n"] == 3
    assert "pw@" not in r["url"] and REDACTED in r["url"]
    assert "sk-123" not in r["hdr"] and r["list"][0]["password"] == REDACTED


def test_crash_record_and_bundle(tmp_path):
    crash = tmp_path / "crashes"
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from syntropy_b200.daemon.bundle import install_crash_handler\n"
            "from syntropy_b200.obs.trace import span\n"
            "install_crash_handler(%r)\n"
            "with span('step', seq=7):\n    pass\n"
            "raise RuntimeError('boom token=abc')\n") % (ROOT, str(crash))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode != 0 and "boom" in r.stderr
    recs = list(crash.iterdir())
    assert len(recs) == 1
    rec = json.loads(recs[0].read_text())
    assert rec["type"] == "RuntimeError" and rec["spans"][-1]["name"] == "step"
    cfg = load_config(env={}, overrides=["model.name=tiny-llama"])
    out = make_bundle(str(tmp_path / "b.tar.gz"), cfg, crash_dir=str(crash))
    with tarfile.open(out) as t:
        names = set(t.getnames())
        assert {"versions.json", "config.json", "env.json", "flight.json", "metrics.prom"} <= names
        assert any(n.startswith("crashes/crash-") for n in names)
        conf = json.load(t.extractfile("config.json"))
        assert conf["config"]["model"]["name"] == "tiny-llama"


def test_repeat_suppression():
    lg = logging.getLogger("syn.test.suppress")
    lg.setLevel(logging.INFO)
    seen = []

    class H(logging.Handler):
        def emit(self, rec):
            seen.append(rec.getMessage())

    h = H()
    f = RepeatSuppressor(window_s=60)
    h.addFilter(f)
    lg.addHandler(h)
    try:
        for _ in range(50):
            lg.info("queue full")
        lg.info("drained")
    finally:
        lg.removeHandler(h)
    assert seen == ["queue full", "drained (previous message repeated 49 times)"]


def test_nvtx_ranges_are_opt_in():
    """SYN_NVTX off: the decorator hands back the function itself; on: a wrapper that still
    returns the function's result (on a host without CUDA it only calls through)."""
    import importlib

    from syntropy_b200.obs import nvtx
    f = lambda x: x + 1  # noqa: E731
    assert nvtx.nvtx_ranged("a")(f) is f or nvtx.ENABLED
    import os
    old = os.environ.get("SYN_NVTX")
    os.environ["SYN_NVTX"] = "1"
    try:
        mod = importlib.reload(nvtx)
        g = mod.nvtx_ranged("a")(f)
        assert g is not f and g(2) == 3
    finally:
        if old is None:
            del os.environ["SYN_NVTX"]
        else:
            os.environ["SYN_NVTX"] = old
        importlib.reload(nvtx)
