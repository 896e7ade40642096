"""Attention for query rows over a prefix of the KV cache (prefill / causal).

Two entry points:

* ``gqa_prefill`` -- the causal prefill kernel (tllm_gqa_prefill): prompt
  rows are cut into blocks of up to 64 consecutive positions of one
  sequence (``prefill_blocks``), and one CTA per (block, query head) streams
  the sequence's K/V tiles once for all 64 rows with tensor-core tiles and a
  causal mask -- the prefill of smollm2_triton/model.py:318-348 (attention at
  :341-343) over the preallocated cache. bf16 caches, head_dim 64 or 128.
* ``gqa_rows`` -- every query row reads the first ``row_len[r]`` cache rows
  of sequence ``row_seq[r]`` with the split-KV decode kernel; it covers the
  other cache precisions and head sizes and the reference's flat-layout
  ``attention_gqa`` (attention_gqa.py:97-119: query i of seq_q sees keys
  j <= seq_k - seq_q + i).
"""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib
from .attention_gqa import DecodeWorkspace, _kv_dtype


def gqa_rows(q_dev, k_cache, v_cache, row_seq_dev, row_len_dev, out_dev, rows,
             n_head, q_row_stride, q_head_stride, out_row_stride, out_head_stride,
             max_len, workspace=None, sm_scale=None, stream=None, keys_hint=0):
    """Low-level wrapper of tllm_gqa_rows (strides in elements). ``out_dev``
    is fp32 or a TLLM_SPLIT buffer (``gpu.split_empty``). ``keys_hint`` > 0
    (the sum of the row lengths, as far as the caller knows it) plans the
    split of each row's keys from that total (tllm_gqa_rows_hint)."""
    Bc, Hkv, S, D = k_cache.shape
    kvd = _kv_dtype(k_cache)
    if workspace is None:
        workspace = DecodeWorkspace(rows, n_head, Hkv, D, S, kvd)
    optr, odt, oplane = gpu.act_args(out_dev)
    args = (q_dev.ptr, int(q_row_stride), int(q_head_stride),
            k_cache.ptr, v_cache.ptr, kvd, _lib.ptr(row_seq_dev),
            _lib.ptr(row_len_dev), optr, odt, oplane, int(out_row_stride),
            int(out_head_stride), int(rows), int(n_head), Hkv, D, Bc, S,
            int(max_len), float(sm_scale or 0.0), workspace.partial.ptr,
            workspace.partial_bytes, workspace.counters.ptr)
    if keys_hint and int(keys_hint) > 0:
        _lib.call("tllm_gqa_rows_hint", *args, int(keys_hint), stream)
    else:
        _lib.call("tllm_gqa_rows", *args, stream)
    return out_dev


PREFILL_BLOCK = 64   # query rows per block of tllm_gqa_prefill


def prefill_blocks(lens, slots=None, row_offsets=None, first_pos=None) -> np.ndarray:
    """Block table of a prefill: prompt i (``lens[i]`` rows starting at row
    ``row_offsets[i]`` of the query / output buffers, default packed one
    after the other) fills cache sequence ``slots[i]`` (default i) from
    position ``first_pos[i]`` (default 0). Returns (n_blocks, 4) int32 rows
    (first row, rows <= 64, cache sequence, first position), blocks with the
    most keys to read first (they take longest)."""
    lens = np.asarray(lens, np.int64).reshape(-1)
    n = len(lens)
    slots = np.arange(n) if slots is None else np.asarray(slots, np.int64).reshape(-1)
    if row_offsets is None:
        row_offsets = np.concatenate([[0], np.cumsum(lens)[:-1]]) if n else np.zeros(0)
    row_offsets = np.asarray(row_offsets, np.int64).reshape(-1)
    first_pos = np.zeros(n, np.int64) if first_pos is None else \
        np.asarray(first_pos, np.int64).reshape(-1)
    out = []
    for i in range(n):
        for j0 in range(0, int(lens[i]), PREFILL_BLOCK):
            out.append((row_offsets[i] + j0, min(PREFILL_BLOCK, int(lens[i]) - j0),
                        slots[i], first_pos[i] + j0))
    blocks = np.array(out, np.int32).reshape(-1, 4)
    if len(blocks):
        work = blocks[:, 3].astype(np.int64) + blocks[:, 1]
        blocks = blocks[np.argsort(-work, kind="stable")]
    return np.ascontiguousarray(blocks)


def prefill_supported(k_cache) -> bool:
    """Whether tllm_gqa_prefill takes this cache (bf16, head_dim 64 / 128)."""
    return _kv_dtype(k_cache) == _lib.BF16 and int(k_cache.shape[3]) in (64, 128)


def gqa_prefill(q_dev, k_cache, v_cache, blocks_dev, n_blocks, out_dev, n_head,
                q_row_stride, q_head_stride, out_row_stride, out_head_stride,
                sm_scale=None, stream=None):
    """Low-level wrapper of tllm_gqa_prefill (strides in elements):
    ``blocks_dev`` holds ``prefill_blocks`` rows on the device; ``out_dev`` is
    fp32 or an operand-format buffer (``gpu.act_empty``)."""
    Bc, Hkv, S, D = k_cache.shape
    optr, odt, oplane = gpu.act_args(out_dev)
    _lib.call("tllm_gqa_prefill", q_dev.ptr, int(q_row_stride), int(q_head_stride),
              k_cache.ptr, v_cache.ptr, _kv_dtype(k_cache), blocks_dev.ptr,
              int(n_blocks), optr, odt, oplane, int(out_row_stride),
              int(out_head_stride), int(n_head), Hkv, D, Bc, S,
              float(sm_scale or 0.0), stream)
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
