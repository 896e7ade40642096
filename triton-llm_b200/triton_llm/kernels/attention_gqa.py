"""GQA attention on sm_100a (drop-in for triton_llm/kernels/attention_gqa.py).

``attention_gqa`` keeps the reference signature, validation and flat layout
(attention_gqa.py:149-269):

    Q: (n_head * seq_q, d_k)   K, V: (n_kv_head * seq_k, d_k)

and head ``h`` reads KV head ``h // (n_head // n_kv_head)``. A single query
row per head (``seq_q == 1``, the decode step) runs the split-KV decode kernel;
several rows (prefill) run the causal prefill kernel.

``gqa_decode`` is the batched decode entry used by the models: it reads the
preallocated cache ``(B, n_kv_head, max_seq, d_k)`` with per-sequence lengths
held on the device, which is the reference's prealloc layout
(smollm2_triton/model.py:219-225) with a leading batch axis.
"""

from __future__ import annotations

import ctypes

import numpy as np

from triton_llm import gpu
from triton_llm import _lib


def _kv_dtype(t) -> int:
    if getattr(t, "is_bf16", False):
        return _lib.BF16
    if t.dtype == np.float32:
        return _lib.F32
    raise ValueError(f"K/V must be float32 or bfloat16, got {t.dtype}")


class DecodeWorkspace:
    """Scratch buffers of the split-KV decode kernel (allocated once).

    ``partial`` holds per-split partial outputs and softmax statistics;
    ``counters`` holds one int per (sequence, query-head group). The kernel
    leaves the counters at zero after every call, so they are cleared once.
    """

    def __init__(self, batch, n_head, n_kv_head, head_dim, max_seq,
                 kv_dtype=_lib.BF16):
        pb, cb = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.call("tllm_gqa_decode_workspace", batch, n_head, n_kv_head,
                  head_dim, max_seq, kv_dtype, ctypes.byref(pb), ctypes.byref(cb))
        self.partial_bytes = pb.value
        self.partial = gpu.allocate((max(pb.value // 4, 1),), np.float32)
        self.counters = gpu.zeros((max(cb.value // 4, 1),), np.int32)
        self.shape = (batch, n_head, n_kv_head, head_dim, max_seq)


def gqa_decode(q_dev, k_cache, v_cache, seq_lens_dev, out_dev, max_len=None,
               workspace: DecodeWorkspace | None = None, sm_scale=None,
               stream=None):
    """Batched split-KV decode attention.

    q_dev       (B, n_head, d) float32
    k_cache     (B, n_kv_head, max_seq, d) float32 or bfloat16
    v_cache     same as k_cache
    seq_lens_dev (B,) int32 on the device, or None (all sequences use max_len)
    out_dev     (B, n_head, d) float32
    """
    B, H, D = q_dev.shape
    Bk, Hkv, S, Dk = k_cache.shape
    if (Bk, Dk) != (B, D) or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError(f"cache shape {k_cache.shape} / {v_cache.shape} does "
                         f"not match q {q_dev.shape}")
    if tuple(out_dev.shape) != (B, H, D):
        raise ValueError(f"out shape {out_dev.shape} != {(B, H, D)}")
    if H % Hkv != 0:
        raise ValueError(f"n_head ({H}) must be divisible by n_kv_head ({Hkv})")
    kvd = _kv_dtype(k_cache)
    if workspace is None:
        workspace = DecodeWorkspace(B, H, Hkv, D, S, kvd)
    _lib.call("tllm_gqa_decode", q_dev.ptr, k_cache.ptr, v_cache.ptr, kvd,
              _lib.ptr(seq_lens_dev), out_dev.ptr, B, H, Hkv, D, S,
              int(max_len or S), float(sm_scale or 0.0), workspace.partial.ptr,
              workspace.partial_bytes, workspace.counters.ptr, stream)
    return out_dev


def attention_gqa(
    q_dev: "gpu.DeviceTensor",
    k_dev: "gpu.DeviceTensor",
    v_dev: "gpu.DeviceTensor",
    n_head: int,
    n_kv_head: int,
    causal: bool = True,
    sm_scale: float | None = None,
) -> "gpu.DeviceTensor":
    """GPU-resident GQA attention. No sync, no host copies.

    Parameters and return value as in the reference
    (triton_llm/kernels/attention_gqa.py:149-187); K/V may also be bfloat16.
    """
    if n_head <= 0:
        raise ValueError(f"n_head must be > 0, got {n_head}")
    if n_kv_head <= 0:
        raise ValueError(f"n_kv_head must be > 0, got {n_kv_head}")
    if n_head % n_kv_head != 0:
        raise ValueError(
            f"n_head ({n_head}) must be divisible by n_kv_head ({n_kv_head})")
    if len(q_dev.shape) != 2 or len(k_dev.shape) != 2 or len(v_dev.shape) != 2:
        raise ValueError(
            f"All inputs must be 2D, got q.ndim={len(q_dev.shape)}, "
            f"k.ndim={len(k_dev.shape)}, v.ndim={len(v_dev.shape)}")
    if q_dev.shape[0] % n_head != 0:
        raise ValueError(
            f"Query shape[0] ({q_dev.shape[0]}) must be divisible by n_head ({n_head})")
    if k_dev.shape[0] % n_kv_head != 0:
        raise ValueError(
            f"Key shape[0] ({k_dev.shape[0]}) must be divisible by n_kv_head ({n_kv_head})")

    d_k = q_dev.shape[1]
    seq_q = q_dev.shape[0] // n_head
    seq_k = k_dev.shape[0] // n_kv_head
    if tuple(k_dev.shape) != (n_kv_head * seq_k, d_k):
        raise ValueError(f"K shape {k_dev.shape} != expected ({n_kv_head * seq_k}, {d_k})")
    if tuple(v_dev.shape) != (n_kv_head * seq_k, d_k):
        raise ValueError(f"V shape {v_dev.shape} != expected ({n_kv_head * seq_k}, {d_k})")

    if seq_q == 0:
        return gpu.allocate((0, d_k), np.float32)
    if seq_k == 0:
        return gpu.zeros((n_head * seq_q, d_k), np.float32)
    if d_k <= 0 or (d_k & (d_k - 1)) != 0:
        raise ValueError(f"d_k ({d_k}) must be a positive power of 2")
    if sm_scale is None:
        sm_scale = 1.0 / (d_k ** 0.5)

    o_dev = gpu.allocate((n_head * seq_q, d_k), np.float32)
    if seq_q == 1:
        # One query row: the causal mask admits every key (abs pos seq_k - 1).
        q3 = gpu.view(q_dev, (1, n_head, d_k))
        k4 = gpu.view(k_dev, (1, n_kv_head, seq_k, d_k))
        v4 = gpu.view(v_dev, (1, n_kv_head, seq_k, d_k))
        o3 = gpu.view(o_dev, (1, n_head, d_k))
        gqa_decode(q3, k4, v4, None, o3, max_len=seq_k, sm_scale=sm_scale)
        return o_dev
    from triton_llm.kernels.attention_prefill import attention_prefill_flat
    attention_prefill_flat(q_dev, k_dev, v_dev, o_dev, n_head, n_kv_head,
                           seq_q, seq_k, d_k, causal, sm_scale)
    return o_dev
