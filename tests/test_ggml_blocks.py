"""GGML block dequantisers against the `gguf` package's reference dequantisation, on random
blocks (every bit pattern of the quants, scales and mins; finite fp16 block scales)."""
import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as T  # noqa: E402
from gguf import quants  # noqa: E402

from syntropy_b200.formats.ggml_blocks import BLOCKS, DEQUANT  # noqa: E402

# byte offsets of fp16 fields per block (randomised to finite values)
FP16_AT = {"Q8_0": [0], "Q4_0": [0], "Q4_1": [0, 2], "Q4_K": [0, 2], "Q6_K": [208]}


@pytest.mark.parametrize("name", ["Q8_0", "Q4_0", "Q4_1", "Q4_K", "Q6_K"])
def test_dequant_matches_gguf(name):
    rng = np.random.default_rng(0)
    n_per, nbytes = BLOCKS[name]
    nb = 64
    raw = rng.integers(0, 256, size=(nb, nbytes), dtype=np.uint8)
    for off in FP16_AT[name]:
        raw[:, off:off + 2] = rng.normal(0, 0.05, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    want = quants.dequantize(raw.reshape(1, -1), getattr(T, name)).reshape(-1)
    got = DEQUANT[name](torch.from_numpy(raw.reshape(-1).copy())).numpy()
    assert got.shape == (nb * n_per,)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", ["Q8_0", "Q4_0", "Q4_1", "Q4_K", "Q6_K"])
def test_native_dequant_matches(name):
    """The C++ block dequantiser (multi-threaded over blocks) equals the PyTorch one and the
    `gguf` package; fp16 scales include subnormals, zeros and negative values."""
    from syntropy_b200._ext import ext
    rng = np.random.default_rng(1)
    n_per, nbytes = BLOCKS[name]
    nb = 5000  # several parallel chunks
    raw = rng.integers(0, 256, size=(nb, nbytes), dtype=np.uint8)
    halves = np.concatenate([rng.normal(0, 0.05, size=nb - 3), [0.0, -0.0, 3e-7]]).astype(np.float16)
    for off in FP16_AT[name]:
        raw[:, off:off + 2] = rng.permutation(halves).view(np.uint8).reshape(nb, 2)
    t = torch.from_numpy(raw.reshape(-1).copy())
    got = ext().ggml_dequant(t, name)
    assert torch.equal(got, DEQUANT[name](t))
    want = quants.dequantize(raw.reshape(1, -1), getattr(T, name)).reshape(-1)
    np.testing.assert_allclose(got.numpy(), want, rtol=1e-6, atol=1e-6)
    with pytest.raises(RuntimeError):
        ext().ggml_dequant(t[:nbytes + 1].contiguous(), name)  # not a whole number of blocks
