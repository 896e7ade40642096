"""Partitioning of a ragged decode batch across GPUs.

Sequences of a decode batch are independent (the reference decodes one
sequence at a time, smollm2_triton/model.py:408-469), so a batch shards
across the GPUs of one box as data-parallel replicas with no collective: each
rank holds its own copy of the weights and the KV caches of its sequences.
A decode step reads every cached key and value once, so a rank's step time
grows with the sum of its sequences' context lengths. ``partition`` balances
that sum with equal sequence counts per rank (longest-processing-time
greedy), computed identically on every rank from the same lengths, so the
ranks need not communicate.
"""

from __future__ import annotations

import numpy as np


def partition(lens, n_parts: int, per_part: int | None = None) -> list[np.ndarray]:
    """Split sequence indices into ``n_parts`` groups of ``per_part``.

    Longest sequence first, each into the group with the smallest total
    length among those not yet full; ties go to the lowest group index.
    Returns one sorted index array per group.
    """
    lens = np.asarray(lens, np.int64)
    n = len(lens)
    if n_parts <= 0:
        raise ValueError(f"n_parts must be positive, got {n_parts}")
    if per_part is None:
        if n % n_parts:
            raise ValueError(f"{n} sequences do not split evenly into {n_parts} parts")
        per_part = n // n_parts
    if per_part * n_parts != n:
        raise ValueError(f"{n_parts} x {per_part} != {n} sequences")
    order = np.argsort(-lens, kind="stable")
    totals = np.zeros(n_parts, np.int64)
    counts = np.zeros(n_parts, np.int64)
    groups: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        open_ = np.flatnonzero(counts < per_part)
        g = open_[np.argmin(totals[open_])]
        groups[g].append(int(i))
        totals[g] += lens[i]
        counts[g] += 1
    return [np.array(sorted(gr), np.int64) for gr in groups]


def ragged_lengths(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    """Context lengths uniform in [lo, hi] from ``np.random.default_rng(seed)``."""
    return np.random.default_rng(seed).integers(lo, hi + 1, n).astype(np.int32)


# ---------------------------------------------------------------------------
# Tensor parallelism by KV head (long-context decode: all ranks serve the same
# sequences, each holds a slice of every layer and of the KV cache).
# ---------------------------------------------------------------------------
def tp_dims(n_head: int, n_kv_head: int, ffn: int, size: int):
    """Per-rank head and FFN counts; rank r holds KV heads
    [r * Hkv/size, (r + 1) * Hkv/size) and exactly the query heads that read
    them (head h reads KV head h // (H / Hkv), attention_gqa.py:76)."""
    if n_kv_head % size or ffn % size:
        raise ValueError(f"{n_kv_head} KV heads / FFN {ffn} do not split over {size} ranks")
    return n_head // size, n_kv_head // size, ffn // size


def shard_llama_layer(w: dict, prefix: str, head_dim: int, n_head: int,
                      n_kv_head: int, ffn: int, rank: int, size: int) -> dict:
    """One layer's HF-layout weights for rank ``rank`` of ``size``:

    q / k / v and gate / up are column-parallel (their output rows are
    sliced), o and down are row-parallel (their input columns are sliced),
    so rank r's o / down outputs are partial sums that an all-reduce
    completes. Norm weights are replicated."""
    H, Hkv, F = tp_dims(n_head, n_kv_head, ffn, size)
    D = head_dim
    q0, k0, f0 = rank * H * D, rank * Hkv * D, rank * F
    p = prefix
    g = lambda k: np.asarray(w[p + k])  # noqa: E731
    return {
        "q": g("self_attn.q_proj.weight")[q0:q0 + H * D],
        "k": g("self_attn.k_proj.weight")[k0:k0 + Hkv * D],
        "v": g("self_attn.v_proj.weight")[k0:k0 + Hkv * D],
        "o": g("self_attn.o_proj.weight")[:, q0:q0 + H * D],
        "gate": g("mlp.gate_proj.weight")[f0:f0 + F],
        "up": g("mlp.up_proj.weight")[f0:f0 + F],
        "down": g("mlp.down_proj.weight")[:, f0:f0 + F],
        "ln1": g("input_layernorm.weight"),
        "ln2": g("post_attention_layernorm.weight"),
    }
