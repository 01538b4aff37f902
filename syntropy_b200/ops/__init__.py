"""Op layer.  On CUDA tensors every op calls its sm_100a kernel in ``syntropy_b200._C``
(raising if the extension is missing); on CPU tensors the same op runs as plain f32
PyTorch, which is what the CPU tests and oracles exercise.

Op names follow the reference's closed op list (crates/kernels/src/op/kind.rs:23-123).
"""
from .core import *  # noqa: F401,F403
