"""Builds the native extension ``syntropy_b200._C`` in-tree.

One shared object holds the C++ runtime (quantisers, Philox, MoE split rule, rings,
format parsers, I/O pool, metrics) and every CUDA kernel.  CUDA code is compiled for
sm_100a only: the ``-gencode`` flag below also stops torch from adding its own arch list.

    python setup.py build_ext --inplace
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


def _sources():
    pats = ["csrc/cpu/*.cpp", "csrc/cuda/*.cu", "csrc/*.cpp"]
    out = []
    for p in pats:
        out += sorted(glob.glob(os.path.join(ROOT, p)))
    return [os.path.relpath(s, ROOT) for s in out]


def _buildinfo():
    import importlib.util
    spec = importlib.util.spec_from_file_location("buildinfo", os.path.join(ROOT, "syntropy_b200", "buildinfo.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.source_hash(ROOT), mod.ABI_VERSION


BUILD_ID, ABI_VERSION = _buildinfo()
# the build identity the loader checks (syn_build_id / syn_abi_version), in a generated header
# that only csrc/cpu/register.cpp includes (rewritten only when it changes)
STAMP_DIR = os.path.join(ROOT, "build", "stamp")
os.makedirs(STAMP_DIR, exist_ok=True)
_stamp = f'#define SYN_BUILD_ID "{BUILD_ID}"\n#define SYN_ABI_VERSION {ABI_VERSION}\n'
_stamp_path = os.path.join(STAMP_DIR, "syn_build_stamp.h")
if not os.path.exists(_stamp_path) or open(_stamp_path).read() != _stamp:
    with open(_stamp_path, "w") as f:
        f.write(_stamp)
CXX_FLAGS = ["-O3", "-std=c++17", "-fno-strict-aliasing", "-Wno-unused-function"]
LIBS = ["rt"]
# Link the shared libstdc++ that torch itself uses.  A toolchain whose libstdc++.so dev link
# does not resolve falls back to libstdc++.a, and a second, static copy of the C++ runtime
# in the process breaks iostream locale facets (formatting a number in an error message
# then crashes).
LINK_FLAGS = ["-l:libstdc++.so.6",
              # export only the module entry point and the C entry points (syn_*)
              "-Wl,--version-script=" + os.path.join(ROOT, "csrc", "exports.map")]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]

setup(
    name="syntropy_b200",
    ext_modules=[
        CUDAExtension(
            name="syntropy_b200._C",
            sources=_sources(),
            include_dirs=[os.path.join(ROOT, "csrc", "include"), os.path.join(ROOT, "csrc"), STAMP_DIR],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
            libraries=LIBS,
            extra_link_args=LINK_FLAGS,
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
