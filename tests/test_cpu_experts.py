"""Host CPU expert tier, without a GPU: the tiled 4-bit GEMV on the CPU (AVX-512 BF16 and plain
C++) against the dequantised f32 product, and the native worker pool driven through its
mailbox exactly as the GPU hand-off kernel drives it (rows, routing CSR, go word), checked
against a plain PyTorch SwiGLU expert FFN."""
import time

import pytest
import torch
import torch.nn.functional as F

from syntropy_b200._ext import ext
from syntropy_b200.ops.core import interleave_gate_up


def _q4(w):
    N, K = w.shape
    rows = ext().q4_quantize_rows_cpu(w.contiguous())
    qw, sm = ext().q4_rows_to_tiled_cpu(rows, N, K)
    return qw, sm, ext().q4_dequant_rows_cpu(rows, N, K).float()


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_cpu_q4t_gemv(mode):
    """mode 0: plain C++, 1: AVX-512 BF16, 2: AVX-512 VNNI (falls back where the ISA is missing)."""
    if mode and not ext().cpu_simd_available():
        pytest.skip("no AVX-512 on this CPU")
    torch.manual_seed(0)
    N, K = 256, 512
    qw, sm, wd = _q4(torch.randn(N, K) * 0.05)
    for R in (1, 3, 6):
        x = torch.randn(R, K).bfloat16()
        ref = x.float() @ wd.t()
        y = ext().cpu_q4t_gemv(qw, sm, x, N, mode)
        assert torch.allclose(y, ref, rtol=1e-4, atol=2e-4 * ref.abs().max().item())


def test_worker_pool_through_mailbox():
    torch.manual_seed(1)
    E, k, H, I, R, n_layers = 8, 2, 256, 128, 4, 2
    layer = 1
    experts = []
    for _ in range(E):
        gu = interleave_gate_up(torch.randn(I, H) * 0.05, torch.randn(I, H) * 0.05)
        experts.append((_q4(gu), _q4(torch.randn(H, I) * 0.05)))
    offs = ext().cpu_mailbox_bytes(E, k, R, H)
    o_off, o_idx, o_pw, o_h, o_pairs, o_out, nbytes = offs
    mb = torch.zeros(nbytes, dtype=torch.uint8)
    w32 = mb.view(torch.int32)
    owned = [1, 4, 6]
    tier = ext().CpuExpertTier(n_layers, E, H, I, k, R, mb.data_ptr(), [], 3, -1)
    for e in owned:
        (qg, sg, _), (qd, sd, _) = experts[e]
        tier.set_expert(layer, e, qg.data_ptr(), sg.data_ptr(), qd.data_ptr(), sd.data_ptr())
    tier.start()
    try:
        for seq in (1, 2):
            h = torch.randn(R, H).bfloat16()
            ids = torch.stack([torch.randperm(E)[:k] for _ in range(R)])
            wts = torch.rand(R, k)
            # routing CSR: pairs sorted by expert, then token
            pairs = sorted((int(ids[t, j]), t, float(wts[t, j])) for t in range(R) for j in range(k))
            tok_off = torch.zeros(E + 1, dtype=torch.int32)
            for e, _, _ in pairs:
                tok_off[e + 1] += 1
            tok_off = torch.cumsum(tok_off, 0).int()
            mb[o_off:o_off + 4 * (E + 1)].view(torch.int32).copy_(tok_off)
            mb[o_idx:o_idx + 4 * R * k].view(torch.int32).copy_(torch.tensor([t for _, t, _ in pairs]).int())
            mb[o_pw:o_pw + 4 * R * k].view(torch.float32).copy_(torch.tensor([w for _, _, w in pairs]))
            mb[o_h:o_h + 2 * R * H].view(torch.bfloat16).copy_(h.reshape(-1))
            w32[1], w32[2] = layer, R
            w32[0] = seq
            t0 = time.time()
            while int(w32[16]) != seq:
                assert time.time() - t0 < 20, "CPU tier did not answer"
                time.sleep(0.001)
            assert int(w32[18]) == 0
            n_out = int(w32[17])
            want = [p for p, (e, _, _) in enumerate(pairs) if e in owned]
            assert n_out == len(want)
            got_pairs = mb[o_pairs:o_pairs + 4 * n_out].view(torch.int32).tolist()
            assert got_pairs == want
            out = mb[o_out:o_out + 4 * n_out * H].view(torch.float32).view(n_out, H)
            for q, p in enumerate(got_pairs):
                e, t, w = pairs[p]
                (_, _, gd), (_, _, dd) = experts[e]
                g = (h[t].float() @ gd.t()).view(I // 8, 2, 8)
                mid = (F.silu(g[:, 0]) * g[:, 1]).reshape(I).bfloat16().float()
                ref = w * (mid @ dd.t())
                assert torch.allclose(out[q], ref, rtol=2e-3, atol=2e-3 * ref.abs().max().item()), (q, e)
        st = tier.stats()
        assert st["jobs"] == 2 and st["pairs"] > 0
    finally:
        tier.stop()


def test_rank_cpus_split_is_disjoint_and_balanced_share():
    from syntropy_b200.experts.cpu_tier import balanced_share, rank_cpus
    allowed = list(range(32))
    w1, l1 = rank_cpus(0, 1, allowed)
    assert w1 == allowed[2:] and l1 == [0, 1]
    parts = [rank_cpus(r, 8, allowed) for r in range(8)]
    workers = [c for w, _ in parts for c in w]
    launch = [c for _, lc in parts for c in lc]
    assert len(set(workers)) == len(workers) == 24 and not set(workers) & set(launch)
    assert all(len(w) == 3 for w, _ in parts)
    # more CPU workers per rank -> a larger CPU share; bounded in (0, 1)
    s8, s2 = balanced_share(3, 8), balanced_share(15, 2)
    assert 0 < s8 < s2 < 1


def test_isa_rates_and_calibrated_family():
    """The host probe of the dot-product instructions and the family the pool uses: a SIMD
    family whenever the host has one (the faster of BF16 and int16 VNNI)."""
    r = ext().cpu_isa_rates(200000)
    assert len(r) == 4 and all(x == -1.0 or x > 0 for x in r)
    mode = ext().cpu_gemv_mode()
    assert mode in (0, 1, 2) and (mode != 0 or not ext().cpu_simd_available())


def test_cpu_pool_bench_runs(monkeypatch, capsys):
    """The pool benchmark drives the mailbox end to end at Qwen3 layer size (two owned
    experts, one layer) and prints one JSON line."""
    import json
    import sys

    from syntropy_b200.bench import cpu_pool
    monkeypatch.setattr(sys, "argv", ["cpu_pool", "--layers", "1", "--threads", "2", "--owned", "2",
                                      "--repeats", "1"])
    cpu_pool.main()
    line = capsys.readouterr().out.strip().splitlines()[-1]
    d = json.loads(line)
    assert d["bench"] == "cpu_expert_pool" and d["threads"] == 2 and d["layer_ms"] > 0


def test_balanced_share_tiers():
    """The CPU share of the host tier balances the pool's rate (per kernel family) against the
    link: one rank alone, 2-4 ranks with the pools capped by shared DRAM, 8 ranks with GPU pairs
    sharing a host link (measured balances: 0.7 on one GPU with 14 int16 workers, ~0.5 at EP2
    with 11 workers)."""
    from syntropy_b200.experts.cpu_tier import balanced_share
    assert balanced_share(14, 1, mode=2) == 0.7
    assert balanced_share(14, 1, mode=1) == 0.6            # the BF16 family is slower per worker
    assert abs(balanced_share(11, 2, mode=2) - 0.51) < 0.01  # DRAM cap, not 11 x 7.5 GB/s
    assert balanced_share(7, 4, mode=2) == balanced_share(7, 2, mode=2)
    assert balanced_share(7, 8, mode=2) > balanced_share(7, 4, mode=2)  # paired links: more to the CPU
    assert 0 < balanced_share(1, 8, mode=2) < balanced_share(15, 1, mode=2) < 1
