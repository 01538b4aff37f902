"""Host enumeration over a recorded /proc + /sys tree: a two-socket host with SMT, two NUMA
nodes (one memory tier each), AVX-512 + AMX, and a GPU whose PCI device sits on node 1."""
import os

from syntropy_b200.probe.host import (cpu_info, isa_level, local_cpus, memory, numa_nodes, parse_cpulist,
                                      pci_numa_node)

V4 = "fpu sse2 cx16 lahf_lm popcnt sse4_1 sse4_2 ssse3 avx avx2 bmi1 bmi2 f16c fma movbe xsave " \
     "avx512f avx512bw avx512cd avx512dq avx512vl avx512_bf16 amx_tile amx_bf16"


def _w(root, path, text):
    p = os.path.join(root, path.lstrip("/"))
    os.makedirs(os.path.dirname(p), exist_ok=True)
    with open(p, "w") as f:
        f.write(text)


def _tree(root):
    # 8 logical CPUs: 2 sockets x 2 cores x 2 threads; cpu c = (socket c // 4, core (c // 2) % 2)
    cpuinfo = "".join(f"processor\t: {c}\nmodel name\t: Test CPU\nflags\t\t: {V4}\n\n" for c in range(8))
    _w(root, "/proc/cpuinfo", cpuinfo)
    for c in range(8):
        _w(root, f"/sys/devices/system/cpu/cpu{c}/topology/physical_package_id", f"{c // 4}\n")
        _w(root, f"/sys/devices/system/cpu/cpu{c}/topology/core_id", f"{(c // 2) % 2}\n")
    _w(root, "/sys/devices/system/node/node0/cpulist", "0-3\n")
    _w(root, "/sys/devices/system/node/node1/cpulist", "4-7\n")
    _w(root, "/sys/devices/system/node/node0/meminfo",
       "Node 0 MemTotal:       104857600 kB\nNode 0 MemFree:         52428800 kB\n")
    _w(root, "/sys/devices/system/node/node1/meminfo",
       "Node 1 MemTotal:       104857600 kB\nNode 1 MemFree:        104857600 kB\n")
    _w(root, "/proc/meminfo", "MemTotal:       209715200 kB\nMemAvailable:   157286400 kB\n"
       "HugePages_Total:      16\nHugepagesize:       2048 kB\n")
    _w(root, "/sys/bus/pci/devices/0000:9b:00.0/numa_node", "1\n")
    _w(root, "/sys/bus/pci/devices/0000:1b:00.0/numa_node", "-1\n")


def test_recorded_host_tree(tmp_path):
    root = str(tmp_path)
    _tree(root)
    c = cpu_info(root)
    assert c == {"model": "Test CPU", "logical_cpus": 8, "physical_cores": 4, "sockets": 2, "isa": "x86-64-v4+amx",
                 "avx512_bf16": True, "amx": True}
    nodes = numa_nodes(root)
    assert [(n["node"], n["cpus"], n["mem_gib"], n["free_gib"]) for n in nodes] == \
        [(0, [0, 1, 2, 3], 100.0, 50.0), (1, [4, 5, 6, 7], 100.0, 100.0)]
    assert memory(root) == {"total_gib": 200.0, "available_gib": 150.0, "hugepages": 16, "hugepage_kib": 2048}
    assert pci_numa_node("0000:9B:00.0", root) == 1 and pci_numa_node("0000:1b:00.0", root) is None
    assert local_cpus(1, root) == [4, 6]                     # one thread per physical core of node 1
    assert local_cpus(1, root, one_per_core=False) == [4, 5, 6, 7]
    assert local_cpus(None, root) == [0, 2, 4, 6]


def test_isa_levels_and_cpulists():
    assert isa_level(set()) == "x86-64"
    assert isa_level({"cx16", "lahf_lm", "popcnt", "sse4_1", "sse4_2", "ssse3"}) == "x86-64-v2"
    assert isa_level(set(V4.split()) - {"avx512vl"}) == "x86-64-v3"
    assert isa_level(set(V4.split()) - {"amx_tile"}) == "x86-64-v4"
    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11] and parse_cpulist("") == []


def test_live_host_report():
    from syntropy_b200.probe import probe_host
    r = probe_host()
    assert r["cpu"]["logical_cpus"] >= 1 and r["cpu"]["isa"].startswith("x86-64")
    assert sum(len(n["cpus"]) for n in r["numa"]) >= 1
