"""fp32 GEMM (drop-in for triton_llm/kernels/gemm.py).

``gemm(h_dev, w_dev, out_dev=None)`` computes ``(M, K) @ (K, N)`` with the
reference's (in, out) weight layout and fp32 accumulation (gemm.py:53-109).
The models use :mod:`triton_llm.kernels.linear` instead, which streams
(out, in) weights through tensor cores with fused epilogues.
"""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib
from ._common import require_f32


def gemm(h_dev: "gpu.DeviceTensor", w_dev: "gpu.DeviceTensor",
         out_dev: "gpu.DeviceTensor | None" = None) -> "gpu.DeviceTensor":
    """GPU-resident GEMM. No sync, no host copies."""
    M, K = h_dev.shape
    K2, N = w_dev.shape
    assert K == K2, f"gemm shape mismatch: ({M},{K}) x ({K2},{N})"
    if out_dev is not None:
        assert tuple(out_dev.shape) == (M, N), \
            f"out_dev shape mismatch: expected ({M},{N}), got {out_dev.shape}"
    if out_dev is None:
        out_dev = gpu.allocate((M, N), np.float32)
    if M == 0 or N == 0:
        return out_dev
    require_f32(h_dev, "h_dev")
    require_f32(w_dev, "w_dev")
    _lib.call("tllm_gemm_f32", h_dev.ptr, w_dev.ptr, out_dev.ptr, M, N, K, None)
    return out_dev
