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
