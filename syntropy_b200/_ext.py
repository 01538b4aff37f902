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
    """Return the native module or raise a RuntimeError naming the build command.  The
    module's ABI version must match this package's; a build from other native sources (a
    stale build) warns, or raises with SYN_STRICT_BUILD=1."""
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        import torch  # noqa: F401  (loads libc10/libtorch that the extension links against)
        mod = importlib.import_module("syntropy_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build state
        _err = e
        raise RuntimeError(
            "syntropy_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"in the repository root ({e})"
        ) from e
    check_build(mod)
    _mod = mod
    return _mod


def check_build(mod) -> str | None:
    """ABI check (fatal) and build-id check (a warning, fatal under SYN_STRICT_BUILD=1)
    against the sources beside this package.  Returns the stale-build message, if any."""
    import os
    import warnings

    from .buildinfo import ABI_VERSION, source_hash
    abi = mod.abi_version() if hasattr(mod, "abi_version") else 0
    if abi != ABI_VERSION:
        raise RuntimeError(f"syntropy_b200._C has ABI version {abi}, this package needs {ABI_VERSION}; rebuild with "
                           "`python setup.py build_ext --inplace`")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if not os.path.isdir(os.path.join(root, "csrc")):
        return None  # installed without sources: nothing to compare with
    want, got = source_hash(root), mod.build_id() if hasattr(mod, "build_id") else "unstamped"
    if want == got:
        return None
    msg = (f"syntropy_b200._C was built from other native sources (build {got}, sources {want}); rebuild with "
           "`python setup.py build_ext --inplace`")
    if os.environ.get("SYN_STRICT_BUILD") == "1":
        raise RuntimeError(msg)
    warnings.warn(msg, RuntimeWarning, stacklevel=3)
    return msg


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
