"""Kernel library (drop-in for triton_llm/kernels/__init__.py).

Every function launches hand-written sm_100a CUDA from libtllm.so; the
reference's names and signatures are kept, and the batched / fused entry
points used by the models are exported next to them.
"""

from .add import add
from .attention import attention
from .attention_gqa import attention_gqa, gqa_decode, DecodeWorkspace
from .attention_prefill import gqa_rows, gqa_prefill, prefill_blocks
from .embedding import embedding, embedding_dev
from .gelu import gelu
from .gemm import gemm
from .layernorm import layer_norm, layer_norm_dev
from .linear import Linear, LinearWorkspace, linear
from .rms_norm import rms_norm
from .rope import precompute_cos_sin, precompute_cos_sin_device, apply_rope
from .softmax import softmax
from .swiglu import swiglu

__all__ = [
    "add",
    "attention",
    "attention_gqa",
    "embedding",
    "gelu",
    "gemm",
    "layer_norm",
    "rms_norm",
    "precompute_cos_sin",
    "apply_rope",
    "softmax",
    "swiglu",
    # batched / fused entry points of the B200 path
    "gqa_decode",
    "gqa_rows",
    "gqa_prefill",
    "prefill_blocks",
    "DecodeWorkspace",
    "embedding_dev",
    "layer_norm_dev",
    "precompute_cos_sin_device",
    "Linear",
    "LinearWorkspace",
    "linear",
]
