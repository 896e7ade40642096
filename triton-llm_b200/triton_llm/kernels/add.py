"""Elementwise add (drop-in for triton_llm/kernels/add.py:54-95)."""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def add(x_dev: "gpu.DeviceTensor", y_dev: "gpu.DeviceTensor",
        out_dev: "gpu.DeviceTensor | None" = None) -> "gpu.DeviceTensor":
    """z = x + y."""
    assert tuple(x_dev.shape) == tuple(y_dev.shape), f"Shape mismatch: {x_dev.shape} vs {y_dev.shape}"
    if out_dev is not None:
        assert tuple(out_dev.shape) == tuple(x_dev.shape), \
            f"out_dev shape mismatch: expected {x_dev.shape}, got {out_dev.shape}"
    N = int(np.prod(x_dev.shape))
    if out_dev is None:
        out_dev = gpu.allocate(x_dev.shape, np.float32)
    if N:
        _lib.call("tllm_elementwise", _lib.EL_ADD, x_dev.ptr, y_dev.ptr, out_dev.ptr, N, None)
    return out_dev
