"""SwiGLU (drop-in for triton_llm/kernels/swiglu.py:70-119)."""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def swiglu(gate_dev: "gpu.DeviceTensor", up_dev: "gpu.DeviceTensor",
           out_dev: "gpu.DeviceTensor | None" = None) -> "gpu.DeviceTensor":
    """out = silu(gate) * up, elementwise."""
    if tuple(gate_dev.shape) != tuple(up_dev.shape):
        raise ValueError(
            f"gate_dev shape {gate_dev.shape} does not match up_dev shape {up_dev.shape}")
    N = int(np.prod(gate_dev.shape))
    if out_dev is not None:
        assert tuple(out_dev.shape) == tuple(gate_dev.shape), \
            f"out_dev shape mismatch: expected {gate_dev.shape}, got {out_dev.shape}"
    if out_dev is None:
        out_dev = gpu.allocate(gate_dev.shape, np.float32)
    if N:
        _lib.call("tllm_elementwise", _lib.EL_SWIGLU, gate_dev.ptr, up_dev.ptr,
                  out_dev.ptr, N, None)
    return out_dev
