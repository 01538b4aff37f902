"""Host enumeration on Linux: CPU model, logical / physical cores, x86-64 ISA level, NUMA nodes
with their CPUs and memory (the host memory tiers, one per NUMA node), hugepages, and the NUMA
node of each GPU's PCI device.  Every path is read under `root` ("/" on a live host; a recorded
tree of `/proc` and `/sys` files in tests).  Reference: crates/probe/src/linux/{cpu.rs,mem.rs,
isa.rs}, crates/probe/src/tiers.rs.
"""
from __future__ import annotations

import os

# x86-64 micro-architecture levels (the psABI's v2 / v3 / v4 feature sets, by /proc/cpuinfo flag)
ISA_LEVELS = [
    ("x86-64-v2", {"cx16", "lahf_lm", "popcnt", "sse4_1", "sse4_2", "ssse3"}),
    ("x86-64-v3", {"avx", "avx2", "bmi1", "bmi2", "f16c", "fma", "movbe", "xsave"}),
    ("x86-64-v4", {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"}),
]


def _read(root: str, path: str) -> str | None:
    try:
        with open(os.path.join(root, path.lstrip("/"))) as f:
            return f.read()
    except OSError:
        return None


def parse_cpulist(s: str) -> list[int]:
    """"0-3,8,10-11" -> [0, 1, 2, 3, 8, 10, 11]"""
    out = []
    for part in s.strip().split(","):
        if not part:
            continue
        a, _, b = part.partition("-")
        out.extend(range(int(a), int(b or a) + 1))
    return out


def isa_level(flags: set[str]) -> str:
    level = "x86-64"
    for name, need in ISA_LEVELS:
        if not need <= flags:
            break
        level = name
    if level == "x86-64-v4" and {"amx_tile", "amx_bf16"} <= flags:
        level += "+amx"
    return level


def cpu_info(root: str = "/") -> dict:
    text = _read(root, "/proc/cpuinfo") or ""
    model, flags = None, set()
    for line in text.splitlines():
        k, _, v = line.partition(":")
        k = k.strip()
        if k == "model name" and model is None:
            model = v.strip()
        elif k == "flags" and not flags:
            flags = set(v.split())
    logical = sorted(int(d[3:]) for d in os.listdir(os.path.join(root, "sys/devices/system/cpu"))
                     if d.startswith("cpu") and d[3:].isdigit()) if os.path.isdir(
        os.path.join(root, "sys/devices/system/cpu")) else []
    cores = set()
    for c in logical:
        pkg = _read(root, f"/sys/devices/system/cpu/cpu{c}/topology/physical_package_id")
        core = _read(root, f"/sys/devices/system/cpu/cpu{c}/topology/core_id")
        if pkg is not None and core is not None:
            cores.add((int(pkg), int(core)))
    return {"model": model, "logical_cpus": len(logical), "physical_cores": len(cores) or None,
            "sockets": len({p for p, _ in cores}) or None, "isa": isa_level(flags),
            "avx512_bf16": "avx512_bf16" in flags, "amx": "amx_tile" in flags}


def numa_nodes(root: str = "/") -> list[dict]:
    """One host memory tier per NUMA node: its CPUs and memory (GiB)."""
    base = os.path.join(root, "sys/devices/system/node")
    if not os.path.isdir(base):
        return []
    out = []
    for d in sorted((d for d in os.listdir(base) if d.startswith("node") and d[4:].isdigit()), key=lambda d: int(d[4:])):
        n = int(d[4:])
        cpus = parse_cpulist(_read(root, f"/sys/devices/system/node/{d}/cpulist") or "")
        total = free = None
        for line in (_read(root, f"/sys/devices/system/node/{d}/meminfo") or "").splitlines():
            parts = line.split()
            if len(parts) >= 4 and parts[2] in ("MemTotal:", "MemFree:"):
                v = int(parts[3]) / 2 ** 20  # kB -> GiB
                total, free = (v, free) if parts[2] == "MemTotal:" else (total, v)
        out.append({"node": n, "cpus": cpus, "mem_gib": round(total, 2) if total is not None else None,
                    "free_gib": round(free, 2) if free is not None else None})
    return out


def memory(root: str = "/") -> dict:
    info = {}
    for line in (_read(root, "/proc/meminfo") or "").splitlines():
        k, _, v = line.partition(":")
        if k in ("MemTotal", "MemAvailable", "HugePages_Total", "Hugepagesize"):
            n = int(v.split()[0])
            info[k] = n
    return {"total_gib": round(info["MemTotal"] / 2 ** 20, 2) if "MemTotal" in info else None,
            "available_gib": round(info["MemAvailable"] / 2 ** 20, 2) if "MemAvailable" in info else None,
            "hugepages": info.get("HugePages_Total", 0), "hugepage_kib": info.get("Hugepagesize")}


def pci_numa_node(bus_id: str, root: str = "/") -> int | None:
    """NUMA node of a PCI device ("0000:1b:00.0"); None when the platform reports none (-1)."""
    s = _read(root, f"/sys/bus/pci/devices/{bus_id.lower()}/numa_node")
    if s is None:
        return None
    n = int(s.strip())
    return n if n >= 0 else None


def gpu_numa_nodes(root: str = "/") -> list[dict]:
    """NUMA node of each visible CUDA device (from its PCI bus id)."""
    try:
        import torch
        if not torch.cuda.is_available():
            return []
        out = []
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            out.append({"device": i, "pci": bus, "numa_node": pci_numa_node(bus, root)})
        return out
    except Exception:
        return []


def local_cpus(node: int | None, root: str = "/", one_per_core: bool = True) -> list[int]:
    """CPUs of a NUMA node (every CPU when `node` is None), one logical CPU per physical core."""
    nodes = numa_nodes(root)
    cpus = next((n["cpus"] for n in nodes if n["node"] == node), None) if node is not None else None
    if cpus is None:
        cpus = sorted(c for n in nodes for c in n["cpus"]) or list(range(os.cpu_count() or 1))
    if not one_per_core:
        return cpus
    seen, out = set(), []
    for c in cpus:
        key = (_read(root, f"/sys/devices/system/cpu/cpu{c}/topology/physical_package_id"),
               _read(root, f"/sys/devices/system/cpu/cpu{c}/topology/core_id"))
        if None in key:
            out.append(c)
        elif key not in seen:
            seen.add(key)
            out.append(c)
    return out


def host_report(root: str = "/") -> dict:
    import resource
    soft, hard = resource.getrlimit(resource.RLIMIT_MEMLOCK) if root == "/" else (None, None)
    return {"cpu": cpu_info(root), "memory": memory(root), "numa": numa_nodes(root),
            "gpus": gpu_numa_nodes(root) if root == "/" else [], "memlock": {"soft": soft, "hard": hard}}
