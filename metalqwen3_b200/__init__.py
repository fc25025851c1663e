"""B200 (sm_100a) fused Qwen3 layer kernels behind the q3cu C ABI.

The product is ``libq3cu.so`` (CUDA kernels + C ABI + the C++ CudaContext,
built from ``csrc/``); ``q3cu`` is its ctypes binding over torch tensors and
``shard`` holds the host logic that splits token rows across GPUs.
"""
from .build import build_library, library_path  # noqa: F401

__all__ = ["build_library", "library_path"]
