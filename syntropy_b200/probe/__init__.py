"""Hardware probes (HBM copy bandwidth, pinned H2D, NVLink peer copy, graph launch cost)
and `doctor` checks.  Feed the planner's HardwareModel (reference: crates/probe)."""
from __future__ import annotations

import os
import platform
import time


def _time_cuda(fn, iters=5):
    import torch
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(iters):
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best * 1e-3


def probe_host(quick: bool = True) -> dict:
    """CPU, ISA level, memory, NUMA host tiers and GPU NUMA affinity (`probe.host`); with
    `quick` off also the host read bandwidth and the CPU expert pool's rate (4-bit expert
    rows per second on the allowed cores, the planner's cpu_expert_gbs)."""
    from .host import host_report
    info = {"platform": platform.platform(), "cpus": os.cpu_count()}
    try:
        info.update(host_report("/"))
    except OSError as e:
        info["error"] = str(e)
    if not quick:
        info.update(probe_cpu_experts())
    return info


def probe_cpu_experts(threads: int | None = None, seconds: float = 1.0) -> dict:
    """Host read bandwidth and the CPU expert kernel's rate: one thread's GB/s of 4-bit weights
    on an expert-sized matrix (2 rows, the decode case), times the worker count (the pool's
    threads run independent experts)."""
    import threading

    import torch

    from .._ext import ext
    e = ext()
    cpus = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(os.cpu_count() or 1))
    threads = threads or max(1, len(cpus) - 2)
    out = {"cpu_threads": threads}
    if not e.cpu_simd_available():
        return out
    out["cpu_read_gbs"] = round(e.cpu_read_gbs(1 << 28, threads, 2), 1)
    N, K = 3072, 4096
    w = torch.randn(N, K) * 0.02
    rows = e.q4_quantize_rows_cpu(w)
    qw, sm = e.q4_rows_to_tiled_cpu(rows, N, K)
    x = torch.randn(2, K).bfloat16()
    nbytes = qw.numel() * 4 + sm.numel() * 2
    e.cpu_q4t_gemv(qw, sm, x, N, -1)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds / 4:
        e.cpu_q4t_gemv(qw, sm, x, N, -1)
        n += 1
    per_thread = n * nbytes / (time.perf_counter() - t0) / 1e9
    out["cpu_expert_gbs_per_thread"] = round(per_thread, 2)
    out["cpu_gemv_mode"] = e.cpu_gemv_mode()
    rates = e.cpu_isa_rates(5_000_000)
    out["isa_ns_per_instr"] = {k: round(v, 3) for k, v in
                               zip(("vdpbf16ps", "vfmadd231ps", "vpdpwssd", "vpdpbusd"), rates) if v >= 0}
    out["cpu_expert_gbs"] = round(min(per_thread * threads, out["cpu_read_gbs"]), 1)
    del threading
    return out


def probe_gpu(quick: bool = True) -> dict:
    import torch
    if not torch.cuda.is_available():
        return {"available": False}
    dev = torch.device("cuda:0")
    p = torch.cuda.get_device_properties(dev)
    out = {"available": True, "name": p.name, "sms": p.multi_processor_count,
           "mem_gb": round(p.total_memory / 1e9, 1), "cc": f"{p.major}.{p.minor}", "count": torch.cuda.device_count()}
    n = (256 if quick else 1024) << 20
    a = torch.empty(n, dtype=torch.uint8, device=dev)
    b = torch.empty_like(a)
    t = _time_cuda(lambda: b.copy_(a))
    out["hbm_copy_gbs"] = round(2 * n / t / 1e9, 1)
    h = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    t = _time_cuda(lambda: a.copy_(h, non_blocking=True))
    out["h2d_gbs"] = round(n / t / 1e9, 1)
    g = torch.cuda.CUDAGraph()
    x = torch.zeros(1, device=dev)
    with torch.cuda.graph(g):
        for _ in range(100):
            x.add_(1)
    t = _time_cuda(g.replay)
    out["graph_kernel_gap_us"] = round(t / 100 * 1e6, 2)
    if torch.cuda.device_count() > 1:
        try:
            c = torch.empty(n, dtype=torch.uint8, device="cuda:1")
            t = _time_cuda(lambda: c.copy_(a))
            out["peer_copy_gbs"] = round(n / t / 1e9, 1)
            s0, s1 = torch.empty(64, dtype=torch.uint8, device=dev), torch.empty(64, dtype=torch.uint8, device="cuda:1")
            t = _time_cuda(lambda: s1.copy_(s0), iters=20)
            out["peer_latency_us"] = round(t * 1e6, 2)  # a small peer copy: the alpha of a hand-off
        except Exception as e:  # pragma: no cover
            out["peer_copy_error"] = str(e)
    return out


def probe_all(quick: bool = True) -> dict:
    return {"host": probe_host(quick), "gpu": probe_gpu(quick), "time": time.time()}


def doctor() -> dict:
    checks = []

    def chk(name, fn):
        try:
            r = fn()
            checks.append({"check": name, "ok": bool(r[0]), "detail": r[1]})
        except Exception as e:
            checks.append({"check": name, "ok": False, "detail": str(e)})

    def ext_loaded():
        from .._ext import ext
        m = ext()
        return True, m.__file__

    def torch_cuda():
        import torch
        return True, f"torch {torch.__version__}, cuda available={torch.cuda.is_available()}"

    def memlock():
        import resource
        soft, hard = resource.getrlimit(resource.RLIMIT_MEMLOCK)
        return True, f"RLIMIT_MEMLOCK soft={soft} hard={hard}"

    def nccl():
        import torch.distributed as d
        return d.is_nccl_available(), "nccl available" if d.is_nccl_available() else "nccl missing"

    chk("native extension", ext_loaded)
    chk("torch", torch_cuda)
    chk("memlock", memlock)
    chk("nccl", nccl)
    return {"checks": checks}
