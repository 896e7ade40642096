"""Single-head attention, numpy in/out (drop-in for
triton_llm/kernels/attention.py:141-216). One head of GQA with n_kv = 1."""

from __future__ import annotations

import numpy as np

from triton_llm import gpu
from .attention_gqa import attention_gqa


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = True) -> np.ndarray:
    assert q.ndim == 2 and k.ndim == 2 and v.ndim == 2
    d_k = q.shape[1]
    seq_q = q.shape[0]
    seq_k = k.shape[0]
    assert k.shape == (seq_k, d_k), f"K shape {k.shape} != {(seq_k, d_k)}"
    assert v.shape == (seq_k, d_k), f"V shape {v.shape} != {(seq_k, d_k)}"
    if causal:
        assert seq_q == seq_k, f"causal requires seq_q == seq_k, got {seq_q} vs {seq_k}"
    assert d_k > 0 and (d_k & (d_k - 1)) == 0, \
        f"d_k ({d_k}) must be a positive power of 2"
    if seq_q == 0 or seq_k == 0:
        return np.empty((seq_q, d_k), dtype=np.float32)
    f = lambda a: gpu.to_device(np.require(a, np.float32, ["C_CONTIGUOUS"]))  # noqa: E731
    o = attention_gqa(f(q), f(k), f(v), 1, 1, causal=causal)
    gpu.synchronize()
    return gpu.to_host(o)
