"""syntropy_b200: a Blackwell-native (sm_100a) LLM inference engine.

Framework layer in PyTorch; hot ops are hand-written sm_100a CUDA kernels in the native
extension ``syntropy_b200._C``; multi-GPU runs one process per GPU over NCCL/NVLink.
"""
__version__ = "0.1.0"

from .models.config import ModelConfig, get_config  # noqa: F401
