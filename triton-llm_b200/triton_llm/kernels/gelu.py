"""tanh-GELU (drop-in for triton_llm/kernels/gelu.py:56-83), numpy in/out."""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def gelu(x: np.ndarray) -> np.ndarray:
    if x.size == 0:
        return np.empty(x.shape, dtype=np.float32)
    x_dev = gpu.to_device(np.require(x, dtype=np.float32, requirements=["C_CONTIGUOUS"]))
    y_dev = gpu.allocate(x.shape, np.float32)
    _lib.call("tllm_elementwise", _lib.EL_GELU, x_dev.ptr, None, y_dev.ptr, x.size, None)
    gpu.synchronize()
    return gpu.to_host(y_dev)
