"""Model-file formats: safetensors round trip through the native header parser, GGUF
header/metadata/tensor parsing with Q4_1 blocks, and the 4-bit quantiser (C++ vs torch)."""
import torch

from syntropy_b200._ext import ext
from syntropy_b200.formats.gguf import GGUFFile, write_gguf
from syntropy_b200.formats.q4 import dequant_rows_ref, quantize_rows_ref
from syntropy_b200.formats.safetensors import SafetensorsFile, load_state_dict, save_file


def test_q4_quantizer_cpp_matches_torch():
    w = torch.randn(64, 256) * 0.02
    assert torch.equal(ext().q4_quantize_rows_cpu(w), quantize_rows_ref(w))
    rows = ext().q4_quantize_rows_cpu(w)
    assert torch.allclose(ext().q4_dequant_rows_cpu(rows, 64, 256), dequant_rows_ref(rows, 64, 256))
    err = (dequant_rows_ref(rows, 64, 256) - w).abs().max()
    assert err < 0.02 * 6 / 15


def test_safetensors_roundtrip(tmp_path):
    t = {"a": torch.randn(3, 5), "b": torch.arange(7, dtype=torch.int32), "c": torch.randn(4).to(torch.bfloat16)}
    w = torch.randn(32, 64)
    t["w.q4"] = ext().q4_quantize_rows_cpu(w)
    p = str(tmp_path / "m.safetensors")
    save_file(t, p, metadata={"q4:w": "32,64", "format": "syn"})
    f = SafetensorsFile(p)
    assert set(f.keys()) == set(t)
    assert torch.equal(f.get("a"), t["a"]) and torch.equal(f.get("b"), t["b"]) and torch.equal(f.get("c"), t["c"])
    assert f.meta["format"] == "syn"
    f.close()
    sd = load_state_dict(p)
    assert torch.allclose(sd["w"], dequant_rows_ref(t["w.q4"], 32, 64))


def test_gguf_roundtrip(tmp_path):
    w = torch.randn(16, 64) * 0.05
    rows = ext().q4_quantize_rows_cpu(w)
    p = str(tmp_path / "m.gguf")
    write_gguf(p, {"blk.0.ffn_up.weight": ("q4_1", (rows, (16, 64))), "output_norm.weight": ("f32", torch.ones(64))},
               meta={"general.architecture": "qwen3moe", "qwen3moe.block_count": 94, "x.ratio": 0.5})
    g = GGUFFile(p)
    assert g.version == 3 and g.meta["general.architecture"] == "qwen3moe" and g.meta["qwen3moe.block_count"] == 94
    assert torch.equal(g.raw("blk.0.ffn_up.weight"), rows)
    assert torch.allclose(g.get("blk.0.ffn_up.weight"), dequant_rows_ref(rows, 16, 64))
    assert torch.equal(g.get("output_norm.weight"), torch.ones(64))
    g.close()
