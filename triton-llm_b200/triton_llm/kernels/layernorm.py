"""LayerNorm (drop-in for triton_llm/kernels/layernorm.py:79-152).

numpy in, numpy out like the reference wrapper; the GPT-2 model calls the
device-resident ``layer_norm_dev``.
"""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def layer_norm_dev(x_dev, g_dev, b_dev, out_dev, eps=1e-5, M=None):
    """LayerNorm of the first M rows of x (all rows by default); the output
    is fp32 or in the tensor-core operand format (``gpu.split_empty``)."""
    N = int(x_dev.shape[-1])
    M = int(x_dev.shape[0]) if M is None else int(M)
    ptr, dt, plane = gpu.act_args(out_dev)
    _lib.call("tllm_layernorm", x_dev.ptr, g_dev.ptr, b_dev.ptr, ptr, dt, plane, M,
              N, float(eps), None)
    return out_dev


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray,
               eps: float = 1e-5) -> np.ndarray:
    if x.ndim < 2:
        raise ValueError(f"LayerNorm expects at least a 2D input, got {x.ndim}D")
    if gamma.ndim != 1 or beta.ndim != 1:
        raise ValueError("gamma and beta must be 1D arrays")
    orig_shape = x.shape
    N = orig_shape[-1]
    if gamma.shape != (N,):
        raise ValueError(f"gamma shape mismatch: expected ({N},), got {gamma.shape}")
    if beta.shape != (N,):
        raise ValueError(f"beta shape mismatch: expected ({N},), got {beta.shape}")
    if N == 0:
        raise ValueError("LayerNorm requires the last dimension N > 0")
    x2 = np.ascontiguousarray(x.reshape(-1, N), dtype=np.float32)
    M = x2.shape[0]
    if M == 0:
        return np.empty(orig_shape, np.float32)
    x_dev = gpu.to_device(x2)
    y_dev = gpu.allocate((M, N), np.float32)
    layer_norm_dev(x_dev, gpu.to_device(np.ascontiguousarray(gamma, np.float32)),
                   gpu.to_device(np.ascontiguousarray(beta, np.float32)), y_dev, eps)
    gpu.synchronize()
    return gpu.to_host(y_dev).reshape(orig_shape)
