"""Repository rules checked on every CPU run (the reference's CI task runner checks the same kinds
of rule: dependency layering, hot-thread lint, orphans; xtask/src/{check_deps.rs,hot_threads.rs,
orphan_rule.rs}):

* layering: a subpackage imports only from its own layer or lower ones (the pure-PyTorch
  oracles `models.reference` and `runtime.sampling_ref` may be imported from anywhere);
* hot path: the functions replayed inside the decode CUDA graph make no host round trip
  (`.item()`, `.tolist()`, `.cpu()`, `.numpy()`, a device synchronize, `print`);
* orphans: every native header is included by some source, every native source is built;
* exports: the built extension exports only `PyInit__C` and `syn_*` symbols;
* sources point at no working notes of the build and no path of the build machine.
"""
import ast
import glob
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "syntropy_b200")

LAYERS = {
    "_ext": 0, "__version__": 0, "core": 0, "formats": 0, "text": 0, "obs": 0, "probe": 0,
    "ops": 1, "kv": 1, "experts": 1, "net": 1, "store": 1, "cluster": 1, "config": 1,
    "models": 2, "parallel": 2, "planner": 2,
    "runtime": 3,
    "api": 4, "daemon": 4, "bench": 4, "testkit": 4,
    "cli": 5,
}
ORACLES = {("models", "reference"), ("runtime", "sampling_ref")}
HOT = {"decode_forward", "_attention_decode", "_attention_decode_mla", "_moe_decode", "_shared_expert", "_lm_head"}
SYNCS = {"item", "tolist", "cpu", "numpy", "synchronize"}


def _imports(path, pkg_parts):
    """(subpackage, module) pairs a file imports from inside the package."""
    for node in ast.walk(ast.parse(open(path).read())):
        if isinstance(node, ast.ImportFrom):
            if node.level:
                base = pkg_parts[:len(pkg_parts) - (node.level - 1)]
                mod = base + (node.module.split(".") if node.module else [])
                if mod:
                    yield mod[0], mod[1] if len(mod) > 1 else None
                else:
                    for a in node.names:
                        yield a.name, None
            elif node.module and node.module.startswith("syntropy_b200."):
                parts = node.module.split(".")[1:]
                yield parts[0], parts[1] if len(parts) > 1 else None


def test_layering():
    bad = []
    for path in glob.glob(os.path.join(PKG, "**", "*.py"), recursive=True):
        rel = os.path.relpath(path, PKG).split(os.sep)
        if len(rel) == 1:
            continue  # package entry points may import anything
        sub = rel[0]
        assert sub in LAYERS, f"subpackage {sub} has no layer"
        for tgt, mod in _imports(path, rel[:-1]):
            if tgt == sub or (tgt, mod) in ORACLES:
                continue
            assert tgt in LAYERS, f"{path}: import of unknown subpackage {tgt}"
            if LAYERS[tgt] > LAYERS[sub]:
                bad.append(f"{os.path.relpath(path, ROOT)} ({sub}, layer {LAYERS[sub]}) imports {tgt} "
                           f"(layer {LAYERS[tgt]})")
    assert not bad, "\n".join(bad)


def test_graph_replayed_functions_make_no_host_round_trip():
    src = open(os.path.join(PKG, "runtime", "runner.py")).read()
    found = set()
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, ast.FunctionDef) and node.name in HOT:
            found.add(node.name)
            for sub in ast.walk(node):
                if isinstance(sub, ast.Call):
                    f = sub.func
                    name = f.attr if isinstance(f, ast.Attribute) else getattr(f, "id", None)
                    assert name not in SYNCS and name != "print", \
                        f"{node.name} line {sub.lineno}: {name}() in a graph-replayed function"
    assert found == HOT, f"hot functions renamed or removed: {HOT - found}"


def test_no_orphan_native_files():
    sources = glob.glob(os.path.join(ROOT, "csrc", "**", "*.c*"), recursive=True)
    text = "".join(open(p).read() for p in sources)
    for h in glob.glob(os.path.join(ROOT, "csrc", "include", "**", "*.h"), recursive=True):
        name = os.path.relpath(h, os.path.join(ROOT, "csrc", "include"))
        others = "".join(open(p).read() for p in glob.glob(os.path.join(ROOT, "csrc", "include", "**", "*.h"),
                                                          recursive=True) if p != h)
        assert f'"{name}"' in text or f'"{name}"' in others or f'"{os.path.basename(name)}"' in text + others, \
            f"header {name} is included nowhere"
    setup = open(os.path.join(ROOT, "setup.py")).read()
    pats = re.findall(r'"(csrc/[^"]+)"', setup)
    built = {os.path.normpath(p) for pat in pats for p in glob.glob(os.path.join(ROOT, pat))}
    for p in sources:
        if p.endswith((".cpp", ".cu")) and os.sep + "native" + os.sep not in p:
            assert os.path.normpath(p) in built, f"{p} is not built"


def test_extension_exports_only_the_module_entry_and_c_api():
    so = glob.glob(os.path.join(PKG, "_C*.so"))
    if not so or shutil.which("nm") is None:
        pytest.skip("extension not built here")
    out = subprocess.run(["nm", "-D", "--defined-only", so[0]], capture_output=True, text=True, check=True).stdout
    names = [ln.split()[-1] for ln in out.splitlines() if ln.strip() and ln.split()[-2] in ("T", "D", "B", "R", "W")]
    stray = [n for n in names if n != "PyInit__C" and not n.startswith("syn_")]
    assert not stray, stray[:10]


def test_sources_point_at_no_working_notes_or_machine_paths():
    notes = ["SUR" + "VEY", "DES" + "IGN.md", "VER" + "DICT", "ADV" + "ICE.md", "BASE" + "LINE.md", "gpu" + "run",
             "/ro" + "ot/"]
    files = [p for pat in ("syntropy_b200/**/*.py", "csrc/**/*.c*", "csrc/**/*.h", "csrc/**/*.cuh", "tests/**/*.py",
                           "bench.py", "__graft_entry__.py", "setup.py")
             for p in glob.glob(os.path.join(ROOT, pat), recursive=True)]
    bad = []
    for p in files:
        for i, line in enumerate(open(p, errors="replace"), 1):
            for n in notes:
                if n in line:
                    bad.append(f"{os.path.relpath(p, ROOT)}:{i}: {n}")
    assert not bad, "\n".join(bad[:20])
