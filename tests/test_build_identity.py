"""Build identity of the native extension: the exported C symbols carry the source hash and
ABI version the loader checks; the built module matches the sources in the tree."""
import ctypes

import pytest

from syntropy_b200 import _ext
from syntropy_b200.buildinfo import ABI_VERSION, source_hash


def test_build_matches_sources_and_abi():
    m = _ext.ext()
    assert m.abi_version() == ABI_VERSION
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    assert m.build_id() == source_hash(root), "rebuild: python setup.py build_ext --inplace"
    lib = ctypes.CDLL(m.__file__)
    lib.syn_build_id.restype = ctypes.c_char_p
    assert lib.syn_build_id().decode() == m.build_id() and lib.syn_abi_version() == ABI_VERSION


def test_abi_mismatch_is_fatal_and_stale_build_warns(monkeypatch):
    class Fake:
        def abi_version(self):
            return ABI_VERSION + 1

        def build_id(self):
            return "0"
    with pytest.raises(RuntimeError, match="ABI"):
        _ext.check_build(Fake())
    Fake.abi_version = lambda self: ABI_VERSION
    with pytest.warns(RuntimeWarning, match="other native sources"):
        assert _ext.check_build(Fake())
    monkeypatch.setenv("SYN_STRICT_BUILD", "1")
    with pytest.raises(RuntimeError, match="other native sources"):
        _ext.check_build(Fake())
