"""Kernel library (drop-in for triton_llm/kernels/__init__.py).

Every function launches hand-written sm_100a CUDA from libtllm.so.
"""

from .attention_gqa import attention_gqa, gqa_decode, DecodeWorkspace

__all__ = [
    "attention_gqa",
    "gqa_decode",
    "DecodeWorkspace",
]
