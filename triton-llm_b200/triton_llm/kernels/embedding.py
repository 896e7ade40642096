"""Token + position embedding (drop-in for triton_llm/kernels/embedding.py).

``embedding`` keeps the reference's numpy-in / numpy-out wrapper
(embedding.py:98-187); ``embedding_dev`` is the device-resident gather the
models use (ids, optional positions and output on the GPU).
"""

from __future__ import annotations

import numpy as np

from triton_llm import gpu, _lib


def embedding_dev(ids_dev, wte, out_dev, wpe_dev=None, pos_dev=None):
    """out[m] = wte[ids[m]] (+ wpe[pos[m]]). ``wte`` is a (V, n) DeviceTensor
    (fp32 or bf16) or a ``Linear`` (the table tied to the lm_head, tiled when
    bf16)."""
    M = int(np.prod(ids_dev.shape))
    if hasattr(wte, "dtype") and hasattr(wte, "K") and hasattr(wte, "w"):
        V, n, ptr, dt = wte.N, wte.K, wte.w.ptr, wte.dtype
    else:
        V, n = wte.shape
        ptr, dt = wte.ptr, (_lib.BF16 if wte.is_bf16 else _lib.F32)
    P = wpe_dev.shape[0] if wpe_dev is not None else 0
    _lib.call("tllm_embedding", ids_dev.ptr, ptr, dt,
              wpe_dev.ptr if wpe_dev is not None else None,
              pos_dev.ptr if pos_dev is not None else None, out_dev.ptr, M, n, V,
              P, None)
    return out_dev


def embedding(token_ids: np.ndarray, weight: np.ndarray, pos_weight: np.ndarray,
              position_offset: int = 0) -> np.ndarray:
    assert token_ids.ndim == 2, f"token_ids must be 2-D, got shape {token_ids.shape}"
    assert weight.ndim == 2, f"weight must be 2-D, got shape {weight.shape}"
    assert pos_weight.ndim == 2, f"pos_weight must be 2-D, got shape {pos_weight.shape}"
    batch, seq_len = token_ids.shape
    vocab_size, n_embd = weight.shape
    max_position, n_embd_pos = pos_weight.shape
    assert n_embd == n_embd_pos, \
        f"Embedding dimension mismatch: weight has {n_embd}, pos_weight has {n_embd_pos}"
    assert seq_len <= max_position, f"seq_len ({seq_len}) exceeds max_position ({max_position})"
    assert position_offset + seq_len <= max_position, \
        f"position_offset ({position_offset}) + seq_len ({seq_len}) exceeds max_position ({max_position})"
    if batch == 0 or seq_len == 0:
        return np.empty((batch, seq_len, n_embd), dtype=np.float32)
    ids = np.ascontiguousarray(token_ids, dtype=np.int32).reshape(-1)
    pos = (np.tile(np.arange(seq_len, dtype=np.int32), batch) + position_offset).astype(np.int32)
    out = gpu.allocate((batch * seq_len, n_embd), np.float32)
    embedding_dev(gpu.to_device(ids),
                  gpu.to_device(np.require(weight, np.float32, ["C_CONTIGUOUS"])), out,
                  gpu.to_device(np.require(pos_weight, np.float32, ["C_CONTIGUOUS"])),
                  gpu.to_device(pos))
    gpu.synchronize()
    return gpu.to_host(out).reshape(batch, seq_len, n_embd)
