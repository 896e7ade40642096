"""Row softmax (drop-in for triton_llm/kernels/softmax.py:105-180)."""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    x = np.require(x, dtype=np.float32, requirements=["C_CONTIGUOUS"])
    if x.size == 0:
        return np.empty(x.shape, dtype=np.float32)
    original_ndim = x.ndim
    if x.ndim not in (1, 2):
        raise NotImplementedError(
            f"softmax on {x.ndim}D input is not implemented (only 1D and 2D are supported)")
    if x.ndim == 1:
        x = x.reshape(1, -1)
    pos_axis = axis if axis >= 0 else original_ndim + axis
    if pos_axis != original_ndim - 1:
        raise NotImplementedError(
            f"softmax along axis={axis} on {original_ndim}D input is not implemented "
            f"(only the last dimension, axis={original_ndim - 1}, is supported)")
    M, N = x.shape
    x_dev = gpu.to_device(x)
    y_dev = gpu.allocate(x.shape, np.float32)
    _lib.call("tllm_softmax", x_dev.ptr, y_dev.ptr, M, N, None)
    gpu.synchronize()
    y = gpu.to_host(y_dev)
    return y.reshape(-1) if original_ndim == 1 else y
