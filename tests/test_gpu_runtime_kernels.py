"""Runtime kernels on the GPU: the bounded doorbell wait runs out on a flag that nothing sets
(error bit, context still usable) and passes once the flag is rung; device timestamps are
monotone; parity taps; K/V page pack / unpack round trip against PyTorch indexing."""
import pytest
import torch

from syntropy_b200 import ops

pytestmark = pytest.mark.gpu


def test_doorbell_times_out_and_context_survives(cuda):
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    waited = torch.zeros(1, dtype=torch.int64, device=cuda)
    ops.doorbell_wait(flag, 5, 0.05, status, waited)  # nothing ever rings: the wait must give up
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    assert int(waited.item()) >= 50_000_000
    # the context is still usable, and a rung flag is seen without an error
    status.zero_()
    ops.doorbell_ring(flag, 5)
    ops.doorbell_wait(flag, 5, 0.05, status, waited)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal((torch.ones(4, device=cuda) * 2).cpu(), torch.full((4,), 2.0))


def test_timestamps_monotone(cuda):
    buf = torch.zeros(3, dtype=torch.int64, device=cuda)
    ops.timestamp(buf, 0)
    torch.cuda._sleep(1_000_000)
    ops.timestamp(buf, 1)
    ops.timestamp(buf, 2)
    t = buf.cpu().tolist()
    assert 0 < t[0] < t[1] <= t[2]


def test_parity_taps(cuda):
    torch.manual_seed(0)
    x = torch.randn(10, 300, device=cuda).to(torch.bfloat16)
    idx = torch.tensor([3, 0, 9], dtype=torch.int32, device=cuda)
    out = torch.empty(3, 300, device=cuda)
    ops.tap_rows(x, idx, out)
    ref = x[idx.long()].float()
    assert torch.equal(out, ref)
    cmp = ops.tap_compare(out + 0.01, ref).cpu()
    assert torch.allclose(cmp[:, 0], torch.full((3,), 0.01), atol=1e-4)
    want = (torch.full((300,), 0.01).norm() / ref.cpu().norm(dim=-1))
    assert torch.allclose(cmp[:, 1], want, rtol=1e-3)


def test_kv_pack_unpack(cuda):
    torch.manual_seed(1)
    kc = torch.randn(12, 4, 16, 128, device=cuda).to(torch.bfloat16)
    vc = torch.randn(12, 4, 16, 128, device=cuda).to(torch.bfloat16)
    pages = torch.tensor([7, 2, 11], dtype=torch.int32, device=cuda)
    packed = ops.kv_pack(kc, vc, pages)
    assert torch.equal(packed[:, 0].reshape(3, 4, 16, 128), kc[pages.long()])
    assert torch.equal(packed[:, 1].reshape(3, 4, 16, 128), vc[pages.long()])
    k2, v2 = torch.zeros_like(kc), torch.zeros_like(vc)
    ops.kv_unpack(packed, k2, v2, pages)
    assert torch.equal(k2[pages.long()], kc[pages.long()]) and torch.equal(v2[pages.long()], vc[pages.long()])
    assert k2[0].abs().sum().item() == 0
