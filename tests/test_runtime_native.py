"""Native host runtime: SPSC rings (in-process and shared memory across processes), the
data-plane frame codec (byte layout + CRC32C), the MoE split rule against a direct
transcription of its definition, the pread I/O pool and the metric histograms."""
import multiprocessing as mp
import os
import random

import torch

from syntropy_b200._ext import ext


def test_spsc_ring_fifo_and_full():
    r = ext().SpscRing(8, 64)
    for i in range(8):
        assert r.push(bytes([i]) * (i + 1))
    assert not r.push(b"x")  # full
    for i in range(8):
        assert r.pop() == bytes([i]) * (i + 1)
    assert r.pop() is None


def _consumer(name, size, n, q):
    e = ext()
    reg = e.ShmRegion(name, size, False)
    r = e.SpscRing(reg.address(), 0, 0, False)
    got = []
    while len(got) < n:
        m = r.pop()
        if m is not None:
            got.append(int.from_bytes(m, "little"))
    q.put(got)


def test_spsc_ring_across_processes():
    e = ext()
    name = f"/syn_test_{os.getpid()}"
    size = e.SpscRing.bytes_needed(64, 16) + 4096
    reg = e.ShmRegion(name, size, True)
    r = e.SpscRing(reg.address(), 64, 16, True)
    ctx = mp.get_context("fork")
    q = ctx.Queue()
    p = ctx.Process(target=_consumer, args=(name, size, 1000, q))
    p.start()
    i = 0
    while i < 1000:
        if r.push(i.to_bytes(8, "little")):
            i += 1
    assert q.get(timeout=60) == list(range(1000))
    p.join(timeout=30)


def test_frame_roundtrip_and_layout():
    e = ext()
    ext_b, pay = b"abc", bytes(range(200))
    f = e.frame_encode(0x01, 0x8, 7, 3, 4, 99, 5, ext_b, pay)
    assert f[:4] == b"SYNF" and f[4] == 1 and f[5] == 0x01
    assert len(f) == 64 + 64 + 200
    assert int.from_bytes(f[48:52], "little") == 64 and int.from_bytes(f[52:56], "little") == 200
    assert int.from_bytes(f[56:60], "little") == e.crc32c(pay)
    rc, spec, x, p = e.frame_decode(f)
    assert rc == 0 and spec["step"] == 99 and spec["chan_seq"] == 5 and spec["instance"] == 7
    assert x[:3] == ext_b and p == pay
    bad = bytearray(f)
    bad[100] ^= 1
    assert e.frame_decode(bytes(bad))[0] == 3  # header CRC covers the extension
    bad = bytearray(f)
    bad[-1] ^= 1
    assert e.frame_decode(bytes(bad))[0] == 4


def test_crc32c_known_value():
    # RFC 3720 (iSCSI) check value for "123456789"
    assert ext().crc32c(b"123456789") == 0xE3069283


def _assign_by_definition(route, eligible, n_experts, b_copy, expert_bytes, copy_slots):
    MISS, HIT, CPU = 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFE
    out = []
    elig = lambda e: e < n_experts and (eligible[e >> 5] >> (e & 31)) & 1  # noqa: E731
    for i, (e, t, slot) in enumerate(route):
        if slot != MISS:
            out.append(HIT)
        elif elig(e):
            c = sum(1 for j, (f, u, s2) in enumerate(route)
                    if s2 == MISS and elig(f) and (u > t or (u == t and (f < e or (f == e and j < i)))))
            ok = c < copy_slots and expert_bytes <= b_copy and (c + 1) * expert_bytes <= b_copy
            out.append(c if ok else CPU)
        else:
            out.append(CPU)
    return out


def test_moe_assign_matches_definition():
    rng = random.Random(0)
    for _ in range(200):
        n_exp = rng.choice([8, 64, 128, 256])
        n = rng.randint(1, 40)
        route = [(rng.randrange(n_exp), rng.randint(1, 9), rng.choice([0xFFFFFFFF, 0xFFFFFFFF, 3])) for _ in range(n)]
        eligible = [rng.getrandbits(32) for _ in range((n_exp + 31) // 32)]
        b_copy, eb, cs = rng.randint(0, 10) * 100, rng.choice([50, 100, 300]), rng.randint(0, 6)
        got = ext().moe_assign(torch.tensor(route, dtype=torch.int64), torch.tensor(
            [x - (1 << 32) if x >= (1 << 31) else x for x in eligible], dtype=torch.int32), n_exp, b_copy, eb, cs)
        assert got.tolist() == _assign_by_definition(route, eligible, n_exp, b_copy, eb, cs)


def test_io_pool_reads_extents(tmp_path):
    data = os.urandom(3 * 4096 + 123)
    p = tmp_path / "blob.bin"
    p.write_bytes(data)
    buf = torch.zeros(len(data), dtype=torch.uint8)
    pool = ext().IoPool(3)
    pool.submit(str(p), 0, 4096, buf.data_ptr())
    pool.submit(str(p), 4096, 2 * 4096 + 123, buf.data_ptr() + 4096)
    assert pool.wait_all() == len(data)
    assert bytes(buf.numpy()) == data


def test_histogram_quantiles():
    h = ext().Histogram()
    for v in range(1, 10001):
        h.record(v)
    assert h.count() == 10000
    q50 = h.quantile(0.5)
    assert 0.85 * 5000 <= q50 <= 5000 * 1.01
    c = ext().Counter()
    c.add(5)
    c.add(7)
    assert c.get() == 12


def test_numa_binding_from_fake_nvml():
    """NUMA CPU set decoded from an NVML affinity bitmask (fake NVML, no GPU)."""
    from syntropy_b200.parallel.dist import numa_cpus

    class FakeNvml:
        def nvmlInit(self):
            pass

        def nvmlDeviceGetHandleByIndex(self, i):
            return i

        def nvmlDeviceGetCpuAffinity(self, h, n):
            return [0b1010] + [0] * (n - 1) if h == 0 else [0, 1] + [0] * max(0, n - 2)

    assert numa_cpus(0, FakeNvml()) == [1, 3]
    import os
    if (os.cpu_count() + 63) // 64 >= 2:
        assert numa_cpus(1, FakeNvml()) == [64]

    class Broken:
        def nvmlInit(self):
            raise RuntimeError("no driver")

    assert numa_cpus(0, Broken()) is None


def test_error_message_with_numbers_raises():
    """A C++ check whose message formats numbers must raise, not crash: the extension has to
    share the process's one C++ runtime (a second, static copy breaks iostream formatting)."""
    import pytest
    import torch
    from syntropy_b200._ext import ext
    with pytest.raises(RuntimeError, match="N=10 K=64"):
        ext().q4_rows_to_tiled_cpu(torch.zeros(10 * 2 * 20, dtype=torch.uint8), 10, 64)


def test_cpu_taps_and_kv_pack():
    """CPU forms of the parity taps and K/V page pack/unpack (same contracts as the kernels)."""
    import torch
    from syntropy_b200 import ops
    x = torch.randn(6, 32)
    idx = torch.tensor([5, 1], dtype=torch.int32)
    out = torch.empty(2, 32)
    ops.tap_rows(x, idx, out)
    assert torch.equal(out, x[[5, 1]])
    assert ops.tap_compare(out, out).abs().max().item() == 0
    kc, vc = torch.randn(5, 2, 16, 8), torch.randn(5, 2, 16, 8)
    pages = torch.tensor([4, 0], dtype=torch.int32)
    packed = ops.kv_pack(kc, vc, pages)
    k2, v2 = torch.zeros_like(kc), torch.zeros_like(vc)
    ops.kv_unpack(packed, k2, v2, pages)
    assert torch.equal(k2[[4, 0]], kc[[4, 0]]) and torch.equal(v2[[4, 0]], vc[[4, 0]])


def test_step_desc_fill_matches_python_views():
    """The native descriptor fill writes the layout the runner's tensor views read; padding
    rows are inert (slot -1, null page, greedy)."""
    import torch
    from syntropy_b200._ext import ext
    from syntropy_b200.runtime.runner import StepDesc
    d = StepDesc(8, 5, torch.device("cpu"))
    ext().step_desc_fill(d.host, 8, 5, [11, 12], [3, 40], [0, 7], [100, 205], [1, 2], [0, 1], [0, 4],
                         [0.0, 0.7], [1.0, 0.9], [[4, 5], [1, 2, 3]], 4)
    h = d.h
    assert h["tokens"][:4].tolist() == [11, 12, 0, 0]
    assert h["pos"][:4].tolist() == [3, 40, 0, 0]
    assert h["ctx_len"][:4].tolist() == [4, 41, 1, 1]
    assert h["slot"][:4].tolist() == [100, 205, -1, -1]
    assert h["top_k"][:2].tolist() == [0, 7] and h["counter"][:2].tolist() == [0, 4]
    assert abs(h["temperature"][1].item() - 0.7) < 1e-6 and abs(h["top_p"][1].item() - 0.9) < 1e-6
    assert h["block_tables"][0, :2].tolist() == [4, 5] and h["block_tables"][1, :3].tolist() == [1, 2, 3]
    assert h["block_tables"][2, 0].item() == 0


def test_arena_and_swap_planner():
    """Native tier pieces: the arena reuses and coalesces ranges; the swap planner pairs the
    coldest resident with the hottest host expert under hysteresis."""
    from syntropy_b200._ext import ext
    a = ext().Arena(1000)
    x = a.alloc(100, 64)
    y = a.alloc(300, 256)
    z = a.alloc(200, 16)
    assert x == 0 and y == 256 and z == 560 and a.used() == 600  # [100, 256) is too small for z
    a.release(y)
    a.release(z)
    assert a.largest_free() == 1000 - 100 and a.alloc(800, 16) == 112
    assert a.alloc(200, 16) == -1
    plan = ext().tier_plan_swaps([1.0, 9.0, 0.5, 7.0, 0.0], [True, False, True, False, True], 5, 1.25)
    assert plan == [(4, 1), (2, 3)]
    assert ext().tier_plan_swaps([5.0, 5.5], [True, False], 3, 1.25) == []
