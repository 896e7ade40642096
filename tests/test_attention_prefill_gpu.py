"""Causal prefill attention kernel (tllm_gqa_prefill) vs the oracle (GPU).

Prompts of a batch fill their cache sequences; every prompt row attends its
own sequence up to its own position (the reference's causal attention_gqa,
triton_llm/kernels/attention_gqa.py:97-119, as the SmolLM2 prefill calls it,
smollm2_triton/model.py:341-343). Cache rows past each block's last
position are poisoned with NaN: the kernel must never let them through.
Tolerance atol 1e-4 (the reference's GQA tolerance); the cache holds bf16
values, so the only difference to the oracle is the order of fp32 sums.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ops

pytestmark = pytest.mark.gpu

ATOL = 1e-4
F32 = np.float32


@pytest.fixture(scope="module")
def gpu():
    from triton_llm import gpu as g
    g._initialize()
    g.device_error(reset=True)
    yield g
    assert g.device_error(reset=True) == 0, "kernel reported a device error"


def _bf16(x):
    return ops.bf16_round(np.asarray(x, F32))


def _case(gpu, H, Hkv, D, lens, first_pos, S, out_kind, seed=0):
    """Prompts ``lens`` starting at ``first_pos`` in cache sequences 0..n-1
    (the rows before first_pos are an earlier chunk already in the cache)."""
    from triton_llm.kernels import gqa_prefill, prefill_blocks
    rng = np.random.default_rng(seed)
    n = len(lens)
    B = n + 1                                   # one extra, untouched sequence
    kc = np.full((B, Hkv, S, D), np.nan, F32)
    vc = np.full((B, Hkv, S, D), np.nan, F32)
    for b in range(n):
        end = first_pos[b] + lens[b]
        kc[b, :, :end] = _bf16(rng.standard_normal((Hkv, end, D), dtype=F32))
        vc[b, :, :end] = _bf16(rng.standard_normal((Hkv, end, D), dtype=F32))
    M = int(sum(lens))
    q = rng.standard_normal((M, H, D), dtype=F32)
    blocks = prefill_blocks(lens, first_pos=first_pos)
    kd, vd = gpu.to_device_bf16(kc), gpu.to_device_bf16(vc)
    qd, bd = gpu.to_device(q), gpu.to_device(blocks)
    if out_kind == "f32":
        od = gpu.allocate((M, H * D), np.float32)
    else:
        od = gpu.act_empty(M, H * D, 2 if out_kind == "split" else 1)
    gqa_prefill(qd, kd, vd, bd, len(blocks), od, H, H * D, D, H * D, D)
    gpu.synchronize()
    got = od.to_numpy() if out_kind == "f32" else gpu.split_to_host(od, M)
    want = np.zeros((M, H, D), F32)
    r = 0
    for b in range(n):
        L, p0 = lens[b], first_pos[b]
        end = p0 + L
        qf = q[r:r + L].transpose(1, 0, 2).reshape(H * L, D)
        kf = kc[b, :, :end].reshape(Hkv * end, D)
        vf = vc[b, :, :end].reshape(Hkv * end, D)
        o = ops.gqa_attention(qf, kf, vf, H, Hkv, causal=True)
        want[r:r + L] = o.reshape(H, L, D).transpose(1, 0, 2)
        r += L
    return got.reshape(M, H, D), want


@pytest.mark.parametrize("H,Hkv,D", [(9, 3, 64), (24, 8, 128), (12, 12, 64),
                                      (8, 2, 128)])
def test_prefill_matches_oracle(gpu, H, Hkv, D):
    lens = [1, 63, 64, 65, 200, 17]
    got, want = _case(gpu, H, Hkv, D, lens, [0] * len(lens), 256, "f32")
    assert np.all(np.isfinite(got))
    np.testing.assert_allclose(got, want, atol=ATOL)


@pytest.mark.parametrize("out_kind", ["split", "bf16"])
def test_prefill_operand_output(gpu, out_kind):
    """Output written in the projection operand format: hi + lo planes hold
    the fp32 result to ~16 bits; one bf16 plane to bf16 rounding."""
    lens = [70, 5, 128]
    got, want = _case(gpu, 9, 3, 64, lens, [0, 0, 0], 192, out_kind, seed=3)
    tol = ATOL if out_kind == "split" else 1e-2
    np.testing.assert_allclose(got, want, atol=tol)


def test_prefill_chunked_start(gpu):
    """Prompts that continue a cached prefix (first position > 0): each row
    also sees the earlier chunk's keys."""
    lens, first = [40, 64, 3, 130], [100, 1, 63, 64]
    got, want = _case(gpu, 24, 8, 128, lens, first, 320, "f32", seed=5)
    np.testing.assert_allclose(got, want, atol=ATOL)


def test_prefill_long_prompt_and_blocks_order(gpu):
    """A 2048-row prompt (32 blocks, up to 32 key tiles each) beside short
    ones; the block table puts the longest blocks first."""
    from triton_llm.kernels import prefill_blocks
    lens = [2048, 33, 1]
    blocks = prefill_blocks(lens)
    work = blocks[:, 3] + blocks[:, 1]
    assert (np.diff(work) <= 0).all() and blocks[:, 1].max() <= 64
    assert int(blocks[:, 1].sum()) == sum(lens)
    got, want = _case(gpu, 9, 3, 64, lens, [0, 0, 0], 2048, "f32", seed=7)
    np.testing.assert_allclose(got, want, atol=ATOL)


def test_prefill_equals_row_path(gpu):
    """The block kernel and the per-row split-KV path agree on the same
    prompts (both against the bf16 cache)."""
    from triton_llm.kernels import gqa_prefill, gqa_rows, prefill_blocks
    rng = np.random.default_rng(9)
    H, Hkv, D, S = 9, 3, 64, 256
    lens = [100, 37]
    kc = _bf16(rng.standard_normal((2, Hkv, S, D), dtype=F32))
    vc = _bf16(rng.standard_normal((2, Hkv, S, D), dtype=F32))
    M = sum(lens)
    q = rng.standard_normal((M, H, D), dtype=F32)
    kd, vd, qd = gpu.to_device_bf16(kc), gpu.to_device_bf16(vc), gpu.to_device(q)
    blocks = prefill_blocks(lens)
    a = gpu.allocate((M, H * D), np.float32)
    gqa_prefill(qd, kd, vd, gpu.to_device(blocks), len(blocks), a, H, H * D, D, H * D, D)
    seq = np.repeat(np.arange(2, dtype=np.int32), lens)
    pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
    b = gpu.allocate((M, H * D), np.float32)
    gqa_rows(qd, kd, vd, gpu.to_device(seq), gpu.to_device(pos + 1), b, M, H, H * D, D,
             H * D, D, max(lens))
    gpu.synchronize()
    np.testing.assert_allclose(a.to_numpy(), b.to_numpy(), atol=2e-5)


def test_prefill_rejects_unsupported(gpu):
    from triton_llm import _lib
    lib = _lib.load()
    # fp32 cache: not this kernel's (the row path covers it)
    st = lib.tllm_gqa_prefill(None, 64, 64, None, None, _lib.F32, None, 1, None,
                              _lib.F32, 0, 64, 64, 1, 1, 64, 1, 64, 0.0, None)
    assert st == _lib.ERR_INVALID_ARG or st == _lib.ERR_UNSUPPORTED
    blocks = gpu.to_device(np.array([[0, 65, 0, 0]], np.int32))   # > 64 rows
    kd = gpu.zeros((1, 1, 128, 64), "bfloat16")
    qd = gpu.zeros((65, 1, 64), np.float32)
    od = gpu.allocate((65, 64), np.float32)
    _lib.call("tllm_gqa_prefill", qd.ptr, 64, 64, kd.ptr, kd.ptr, _lib.BF16, blocks.ptr,
              1, od.ptr, _lib.F32, 0, 64, 64, 1, 1, 64, 1, 128, 0.0, None)
    assert gpu.device_error(reset=True) & 2      # the block was refused on the device
