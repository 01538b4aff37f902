"""Diagnostics: crash records and a redacted diagnostic bundle.

`install_crash_handler(dir)` writes one JSON record per uncaught exception (traceback, time,
the last spans of the flight recorder).  `make_bundle(path, cfg)` packs what a bug report
needs into one .tar.gz: resolved config with origins, versions, the probe report, metrics, the
flight recorder, SYN_* environment and the crash records — every value whose key looks like a
credential replaced by "<redacted>".
Reference: crates/daemon/src/{bundle.rs,bundle/redact.rs,crash.rs} (bundle with redaction,
crash records)."""
from __future__ import annotations

import io
import json
import os
import re
import sys
import tarfile
import time
import traceback

_SECRET = re.compile(r"(token|secret|password|passwd|api[_-]?key|credential|private|auth)", re.I)
REDACTED = "<redacted>"


def redact(obj, key: str = ""):
    """Copy of a JSON-like value with credential-like keys' values replaced."""
    if key and _SECRET.search(key):
        return REDACTED
    if isinstance(obj, dict):
        return {k: redact(v, str(k)) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [redact(v) for v in obj]
    if isinstance(obj, str):
        # inline credentials in URLs and "Bearer ..." headers
        obj = re.sub(r"(https?://)[^/@\s]+@", r"\1" + REDACTED + "@", obj)
        obj = re.sub(r"(?i)(bearer\s+)\S+", r"\1" + REDACTED, obj)
    return obj


def install_crash_handler(directory: str):
    """Uncaught exceptions leave `crash-<time>-<pid>.json` in `directory` (then the default
    handler runs)."""
    os.makedirs(directory, exist_ok=True)
    prev = sys.excepthook

    def hook(tp, val, tb):
        try:
            from ..obs.trace import FLIGHT
            rec = {"time": time.time(), "pid": os.getpid(), "type": tp.__name__, "message": str(val),
                   "traceback": traceback.format_exception(tp, val, tb), "spans": FLIGHT.dump()[-64:]}
            with open(os.path.join(directory, f"crash-{int(time.time())}-{os.getpid()}.json"), "w") as f:
                json.dump(redact(rec), f, default=str)
        finally:
            prev(tp, val, tb)

    sys.excepthook = hook
    return hook


def _versions() -> dict:
    out = {"python": sys.version.split()[0]}
    try:
        import torch
        out["torch"] = torch.__version__
        out["cuda_runtime"] = torch.version.cuda
        out["cuda_available"] = torch.cuda.is_available()
    except Exception as e:  # noqa: BLE001
        out["torch"] = f"unavailable: {e}"
    try:
        from .. import __version__
        out["syntropy_b200"] = __version__
    except Exception:  # noqa: BLE001
        pass
    return out


def make_bundle(path: str, cfg=None, crash_dir: str | None = None, include_probe: bool = False) -> str:
    """Writes the bundle to `path` (.tar.gz) and returns it."""
    from ..obs.metrics import METRICS
    from ..obs.trace import FLIGHT
    files = {
        "versions.json": _versions(),
        "config.json": redact({"config": cfg.to_dict(), "origin": cfg.origin}) if cfg is not None else {},
        "env.json": redact({k: v for k, v in os.environ.items() if k.startswith("SYN_")}),
        "flight.json": redact(FLIGHT.dump()),
    }
    if include_probe:
        try:
            from ..probe import doctor
            files["doctor.json"] = doctor()
        except Exception as e:  # noqa: BLE001
            files["doctor.json"] = {"error": str(e)}
    with tarfile.open(path, "w:gz") as tar:
        def add(name, data: bytes):
            ti = tarfile.TarInfo(name)
            ti.size = len(data)
            ti.mtime = int(time.time())
            tar.addfile(ti, io.BytesIO(data))
        for name, obj in files.items():
            add(name, json.dumps(obj, indent=2, default=str).encode())
        add("metrics.prom", METRICS.prometheus().encode())
        if crash_dir and os.path.isdir(crash_dir):
            for fn in sorted(os.listdir(crash_dir)):
                if fn.startswith("crash-") and fn.endswith(".json"):
                    with open(os.path.join(crash_dir, fn), "rb") as f:
                        add("crashes/" + fn, f.read())
    return path
