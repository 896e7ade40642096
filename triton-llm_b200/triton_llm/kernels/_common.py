"""Shared helpers of the kernel wrappers."""

from __future__ import annotations

import numpy as np

from triton_llm import gpu


def require_f32(t, name):
    if getattr(t, "is_bf16", False) or t.dtype != np.float32:
        raise ValueError(f"{name} must be float32, got "
                         f"{'bfloat16' if getattr(t, 'is_bf16', False) else t.dtype}")


def upload_f32(arr):
    return gpu.to_device(np.require(arr, dtype=np.float32, requirements=["C_CONTIGUOUS"]))
