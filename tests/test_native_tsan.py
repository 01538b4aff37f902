"""Race detection for the native runtime (host side): the SPSC ring and the CPU expert worker
pool, driven through their real protocols, built with -fsanitize=thread.  A data race makes
ThreadSanitizer print a report and fail the run; a lost wake-up shows as a bounded-wait
failure."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_runtime_under_thread_sanitizer():
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "tsan_runtime")
        cmd = [cxx, "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-pthread", "-I", os.path.join(ROOT, "csrc/include"),
               os.path.join(ROOT, "tests/native/tsan_runtime.cpp"), "-o", exe]
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
        if r.returncode != 0 and "tsan" in (r.stderr or "").lower():
            pytest.skip("ThreadSanitizer runtime not available: " + r.stderr[-300:])
        assert r.returncode == 0, r.stderr[-3000:]
        env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66")
        run = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
        out = run.stdout + run.stderr
        assert "ThreadSanitizer" not in out, out[-4000:]
        assert run.returncode == 0, out[-4000:]
        assert "pool ok" in run.stdout
