"""Build identity of the native extension: a hash over the native sources and the ABI
version of the Python <-> extension interface.  `setup.py` stamps both into the shared object
(`syn_build_id`, `syn_abi_version`); the loader (`_ext.py`) compares them with the sources
beside it, the way the reference's provider loader checks a module's build id and ABI before
using it (crates/kernels-loader/src/module.rs:67)."""
from __future__ import annotations

import glob
import hashlib
import os

# Raised whenever an op's signature or a shared struct changes meaning.
ABI_VERSION = 2

_PATTERNS = ("csrc/**/*.cpp", "csrc/**/*.cu", "csrc/**/*.h", "csrc/**/*.cuh", "csrc/exports.map")


def source_hash(root: str) -> str:
    """BLAKE2b-64 over the native sources (sorted relative paths and contents)."""
    h = hashlib.blake2b(digest_size=8)
    files = sorted({os.path.relpath(p, root) for pat in _PATTERNS
                    for p in glob.glob(os.path.join(root, pat), recursive=True)})
    for rel in files:
        h.update(rel.encode())
        with open(os.path.join(root, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()
