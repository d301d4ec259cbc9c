"""airllm_b200 -- B200-native (sm_100a) GPT-OSS mixture-of-experts block.

The product is the CUDA library libamoe.so behind the C ABI in include/amoe.h
(built in-tree by airllm_b200/build.py).  This package holds its Python
binding (``moe``) and the seeded synthetic workloads (``workloads``).
"""
from .moe import AmoeError, MoEBlock, load_library  # noqa: F401

__all__ = ["AmoeError", "MoEBlock", "load_library"]
