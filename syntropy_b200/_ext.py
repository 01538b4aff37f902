"""Loader for the native extension.

The extension is built in-tree (``python setup.py build_ext --inplace``).  CPU-only code
paths (tests, oracles) can run without it; every CUDA op calls :func:`ext` and raises if
the extension is missing, so a GPU run never silently falls back to eager PyTorch.
"""
from __future__ import annotations

import importlib

_mod = None
_err: Exception | None = None


def ext():
    """Return the native module or raise a RuntimeError naming the build command."""
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        import torch  # noqa: F401  (loads libc10/libtorch that the extension links against)
        _mod = importlib.import_module("syntropy_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build state
        _err = e
        raise RuntimeError(
            "syntropy_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"in the repository root ({e})"
        ) from e
    return _mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
