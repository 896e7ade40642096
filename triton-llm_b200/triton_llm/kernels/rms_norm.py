"""RMSNorm (drop-in for triton_llm/kernels/rms_norm.py:68-115).

``rms_norm`` keeps the reference signature (fp32 device tensors);
``rms_norm_rows`` is the model entry: the first M rows of x, output fp32 or
in the tensor-core operand format (``gpu.split_empty``).
"""

from __future__ import annotations

from triton_llm import gpu, _lib


def rms_norm(x_dev: "gpu.DeviceTensor", w_dev: "gpu.DeviceTensor",
             out_dev: "gpu.DeviceTensor", eps: float = 1e-5) -> "gpu.DeviceTensor":
    """y = (x / sqrt(mean(x^2) + eps)) * w over the last dimension."""
    M, N = x_dev.shape
    assert tuple(w_dev.shape) == (N,), f"w_dev shape mismatch: expected ({N},), got {w_dev.shape}"
    assert tuple(out_dev.shape) == (M, N), \
        f"out_dev shape mismatch: expected ({M},{N}), got {out_dev.shape}"
    if M == 0:
        return out_dev
    if N == 0:
        raise ValueError("RMSNorm requires the last dimension N > 0")
    _lib.call("tllm_rmsnorm", x_dev.ptr, w_dev.ptr, out_dev.ptr, _lib.F32, M, M, N,
              float(eps), None)
    return out_dev


def rms_norm_rows(x_dev, w_dev, out_dev, M: int, eps: float = 1e-5, stream=None):
    N = int(x_dev.shape[-1])
    ptr, dt, plane = gpu.act_args(out_dev)
    _lib.call("tllm_rmsnorm", x_dev.ptr, w_dev.ptr, ptr, dt, plane, int(M), N,
              float(eps), stream)
    return out_dev


def rms_norm_add_rows(h_dev, add_dev, w_dev, out_dev, M: int, eps: float = 1e-5,
                      stream=None):
    """h += add (first M rows, in place), then out = RMSNorm(h)."""
    N = int(h_dev.shape[-1])
    ptr, dt, plane = gpu.act_args(out_dev)
    _lib.call("tllm_rmsnorm_add", h_dev.ptr, add_dev.ptr, w_dev.ptr, ptr, dt, plane,
              int(M), N, float(eps), stream)
    return out_dev


def rms_norm_p2p_rows(h_dev, peer, w_dev, out_dev, M: int, eps: float = 1e-5,
                      stream=None):
    """h += the sum over the peer group of the rows that the last SCATTER
    projection sent (first M rows, in place, rank order), then
    out = RMSNorm(h). ``peer`` is a ``triton_llm.tp.PeerGroup``."""
    N = int(h_dev.shape[-1])
    ptr, dt, plane = gpu.act_args(out_dev)
    _lib.call("tllm_rmsnorm_p2p", h_dev.ptr, peer.ctx, w_dev.ptr, ptr, dt, plane,
              int(M), N, float(eps), stream)
    return out_dev
