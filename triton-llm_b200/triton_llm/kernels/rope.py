"""RoPE (drop-in for triton_llm/kernels/rope.py).

``precompute_cos_sin`` builds the fp32 tables on the host exactly as the
reference does (rope.py:110-121: float32 positions and pair indices, numpy
cos/sin of their outer product); ``apply_rope`` rotates rows in place on the
GPU. In the decode step the rotation is fused into the QKV projection
epilogue (see kernels.linear), which writes K straight into the cache.
"""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def precompute_cos_sin(max_seq_len: int, d_k: int, theta: float = 100000.0):
    """Tables (max_seq_len, d_k // 2) float32: cos/sin(p * theta^(-2i/d_k))."""
    if max_seq_len < 1:
        raise ValueError(f"max_seq_len must be >= 1, got {max_seq_len}")
    if d_k < 2 or d_k % 2 != 0:
        raise ValueError(f"d_k must be even and >= 2, got {d_k}")
    if theta <= 0:
        raise ValueError(f"theta must be > 0, got {theta}")
    half = d_k // 2
    positions = np.arange(max_seq_len, dtype=np.float32)
    indices = np.arange(half, dtype=np.float32)
    freqs = 1.0 / (theta ** (2 * indices / d_k))
    angles = np.outer(positions, freqs)
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


def precompute_cos_sin_device(max_seq_len: int, d_k: int, theta: float = 100000.0):
    c, s = precompute_cos_sin(max_seq_len, d_k, theta)
    return gpu.to_device(c), gpu.to_device(s)


def apply_rope(x_dev: "gpu.DeviceTensor", cos_dev: "gpu.DeviceTensor",
               sin_dev: "gpu.DeviceTensor", seq_len: int,
               position_offset: int = 0) -> "gpu.DeviceTensor":
    """In-place RoPE of x (n_rows, d_k); row r at (r % seq_len) + offset."""
    n_rows, d_k = x_dev.shape
    if d_k < 2 or d_k % 2 != 0:
        raise ValueError(f"d_k must be even and >= 2, got {d_k}")
    half = d_k // 2
    if len(cos_dev.shape) != 2 or len(sin_dev.shape) != 2:
        raise ValueError("cos_dev and sin_dev must be 2D tensors")
    if tuple(cos_dev.shape) != tuple(sin_dev.shape):
        raise ValueError(f"cos_dev and sin_dev shape mismatch: {cos_dev.shape} vs {sin_dev.shape}")
    if cos_dev.shape[1] != half:
        raise ValueError(f"cos_dev last dim must be d_k // 2 ({half}), got {cos_dev.shape[1]}")
    if n_rows == 0:
        return x_dev
    if seq_len < 1:
        raise ValueError(f"seq_len must be >= 1, got {seq_len}")
    if position_offset < 0:
        raise ValueError(f"position_offset must be >= 0, got {position_offset}")
    if position_offset + seq_len > cos_dev.shape[0]:
        raise ValueError(
            f"position_offset ({position_offset}) + seq_len ({seq_len}) "
            f"exceeds cos/sin table size ({cos_dev.shape[0]})")
    if n_rows % seq_len != 0:
        raise ValueError(f"Total rows ({n_rows}) must be a multiple of seq_len ({seq_len})")
    _lib.call("tllm_rope", x_dev.ptr, cos_dev.ptr, sin_dev.ptr, n_rows, d_k,
              int(seq_len), int(position_offset), None)
    return x_dev
