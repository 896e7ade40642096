"""Attention for query rows over a prefix of the KV cache (prefill / causal).

Every query row reads the first ``row_len[r]`` cache rows of sequence
``row_seq[r]``, which expresses causal prefill attention over the
preallocated cache (smollm2_triton/model.py:332-343) and the causal branch of
the reference's flat-layout ``attention_gqa`` (attention_gqa.py:97-119: query
i of seq_q sees keys j <= seq_k - seq_q + i). It runs the same split-KV
kernel as the decode step.
"""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib
from .attention_gqa import DecodeWorkspace, _kv_dtype


def gqa_rows(q_dev, k_cache, v_cache, row_seq_dev, row_len_dev, out_dev, rows,
             n_head, q_row_stride, q_head_stride, out_row_stride, out_head_stride,
             max_len, workspace=None, sm_scale=None, stream=None):
    """Low-level wrapper of tllm_gqa_rows (strides in elements). ``out_dev``
    is fp32 or a TLLM_SPLIT buffer (``gpu.split_empty``)."""
    Bc, Hkv, S, D = k_cache.shape
    kvd = _kv_dtype(k_cache)
    if workspace is None:
        workspace = DecodeWorkspace(rows, n_head, Hkv, D, S, kvd)
    optr, odt, oplane = gpu.act_args(out_dev)
    _lib.call("tllm_gqa_rows", q_dev.ptr, int(q_row_stride), int(q_head_stride),
              k_cache.ptr, v_cache.ptr, kvd, _lib.ptr(row_seq_dev),
              _lib.ptr(row_len_dev), optr, odt, oplane, int(out_row_stride),
              int(out_head_stride), int(rows), int(n_head), Hkv, D, Bc, S,
              int(max_len), float(sm_scale or 0.0), workspace.partial.ptr,
              workspace.partial_bytes, workspace.counters.ptr, stream)
    return out_dev


def attention_prefill_flat(q_dev, k_dev, v_dev, o_dev, n_head, n_kv_head, seq_q,
                           seq_k, d_k, causal, sm_scale):
    """Flat head-major Q (n_head*seq_q, d) / K, V (n_kv*seq_k, d) -> o_dev."""
    kc = gpu.view(k_dev, (1, n_kv_head, seq_k, d_k))
    vc = gpu.view(v_dev, (1, n_kv_head, seq_k, d_k))
    i = np.arange(seq_q, dtype=np.int64)
    if causal:
        lens = np.clip(seq_k - seq_q + i + 1, 0, seq_k).astype(np.int32)
    else:
        lens = np.full(seq_q, seq_k, np.int32)
    seq = gpu.zeros((seq_q,), np.int32)
    ln = gpu.to_device(lens)
    gqa_rows(q_dev, kc, vc, seq, ln, o_dev, seq_q, n_head, d_k, seq_q * d_k,
             d_k, seq_q * d_k, seq_k, sm_scale=sm_scale)
    return o_dev
