"""Packs: aligned extents with a BLAKE3 sidecar, read back through the native I/O pool (O_DIRECT
when aligned); corruption and shape mismatches are refused.  (The expert host tier's save and reload runs
in tests/test_gpu_expert_prefetch.py: the tier exists on GPUs only.)"""
import os

import pytest
import torch

from syntropy_b200.store.pack import ALIGN, read_pack_into, read_sidecar, write_pack


def test_round_trip_and_alignment(tmp_path):
    torch.manual_seed(0)
    ts = {"a": torch.randn(1000), "b": torch.randint(0, 255, (4096 * 3 + 5,), dtype=torch.uint8),
          "c": torch.randn(7, 33).to(torch.bfloat16), "d": torch.arange(12, dtype=torch.int32).view(3, 4)}
    p = str(tmp_path / "w.pack")
    side = write_pack(p, ts)
    assert all(e["offset"] % ALIGN == 0 for e in side["extents"].values())
    assert os.path.getsize(p) % ALIGN == 0
    out = {k: torch.empty_like(v) for k, v in ts.items()}
    n = read_pack_into(p, out, threads=3)
    assert n == sum(v.numel() * v.element_size() for v in ts.values())
    assert all(torch.equal(out[k], ts[k]) for k in ts)
    assert read_sidecar(p)["extents"]["c"]["shape"] == [7, 33]


def test_corruption_and_mismatch_refused(tmp_path):
    p = str(tmp_path / "w.pack")
    write_pack(p, {"a": torch.ones(5000)})
    with open(p, "r+b") as f:
        f.seek(100)
        f.write(b"\x01")
    with pytest.raises(ValueError, match="digest"):
        read_pack_into(p, {"a": torch.empty(5000)})
    with pytest.raises(ValueError, match="target"):
        read_pack_into(p, {"a": torch.empty(4999)}, verify=False)
