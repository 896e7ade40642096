"""Data-parallel partitioning of a ragged decode batch (CPU, incl. a
world-size-2 gloo run of the per-rank selection the bench uses)."""

from __future__ import annotations

import os

import numpy as np
import pytest

from triton_llm import shard


@pytest.mark.parametrize("n_parts", [1, 2, 4, 8])
def test_partition_covers_and_balances(n_parts):
    lens = shard.ragged_lengths(64 * n_parts, 1024, 8192, 4)
    parts = shard.partition(lens, n_parts, 64)
    allidx = np.concatenate(parts)
    assert sorted(allidx.tolist()) == list(range(64 * n_parts))
    assert all(len(p) == 64 for p in parts)
    totals = np.array([lens[p].sum() for p in parts])
    # LPT with equal counts: spread below the longest single context
    assert totals.max() - totals.min() <= lens.max()


def test_partition_first_part_is_n1_workload():
    """With one part the workload is the first 64 draws of the stream, and
    those draws do not depend on how many ranks there are."""
    a = shard.ragged_lengths(64, 1024, 8192, 4)
    b = shard.ragged_lengths(64 * 8, 1024, 8192, 4)
    np.testing.assert_array_equal(a, b[:64])
    assert (a >= 1024).all() and (a <= 8192).all()


def test_partition_rejects_bad_counts():
    with pytest.raises(ValueError):
        shard.partition(np.ones(10), 3)
    with pytest.raises(ValueError):
        shard.partition(np.ones(10), 2, 4)
    with pytest.raises(ValueError):
        shard.partition(np.ones(4), 0)


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lens = shard.ragged_lengths(64 * world, 1024, 8192, 4)
    mine = shard.partition(lens, world, 64)[rank]
    t = torch.tensor(mine, dtype=torch.int64)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    tot = torch.tensor([float(lens[mine].sum())], dtype=torch.float64)
    dist.all_reduce(tot)
    dist.destroy_process_group()
    if rank == 0:
        q.put((sorted(torch.cat(out).tolist()), float(tot.item()), float(lens.sum())))


def test_two_ranks_select_disjoint_shards():
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    idx, tot, want = got
    assert idx == list(range(128))
    assert tot == want


def test_weight_tiling_round_trip():
    """TLLM_BF16_TILED layout: tile (n // 128, k // 64) is one contiguous
    block of 128 x 64 elements; N padded with zero rows."""
    from triton_llm.kernels.linear import tile_bf16, untile_bf16
    rng = np.random.default_rng(0)
    for N, K in ((200, 192), (128, 64), (5, 64)):
        bits = rng.integers(0, 65535, (N, K)).astype(np.uint16)
        flat = tile_bf16(bits)
        n_pad = -(-N // 128) * 128
        assert flat.size == n_pad * K
        np.testing.assert_array_equal(untile_bf16(flat, N, K), bits)
        k_chunks = K // 64
        for (n, k) in ((0, 0), (N - 1, K - 1), (min(N - 1, 130), 65 % K)):
            idx = ((n // 128) * k_chunks + k // 64) * 8192 + (n % 128) * 64 + k % 64
            assert flat[idx] == bits[n, k]
