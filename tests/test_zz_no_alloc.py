"""The allocation-free decode entry point (tllm_gqa_decode_noalloc).

Some callers of this library cannot let it allocate device memory: servers
that split all of HBM into their own arenas, hosts that forbid hidden
allocations, decode loops that must not block in cudaMalloc. For them
tllm_gqa_decode_noalloc takes its split-KV scratch from a fixed device array
inside libtllm.so. This test calls it through the C ABI and checks that two
calls in a row give the same result as the allocating entry point
(tllm_gqa_decode with caller-owned scratch), within the attention tests'
tolerance, and that an over-limit batch is refused before any launch.

The file name makes pytest collect it last; it sets up everything it uses,
so it also passes when run alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import inputs
from oracle import ops

pytestmark = pytest.mark.gpu

ATOL = 1e-4  # tests/test_attention_decode_gpu.py


def test_noalloc_matches_allocating_entry_point():
    from triton_llm import _lib, gpu
    from triton_llm.kernels import DecodeWorkspace, gqa_decode

    gpu._initialize()
    lib = _lib.load()
    B, H, Hkv, D, S = 24, 9, 3, 64, 2048
    lens, q, ks, vs = inputs.cfg2_inputs(batch=B)
    kc = inputs.pack_cache(ks, S)
    vc = inputs.pack_cache(vs, S)
    qd = gpu.to_device(q)
    kd = gpu.to_device_bf16(kc)
    vd = gpu.to_device_bf16(vc)
    ld = gpu.to_device(lens)
    ws = DecodeWorkspace(B, H, Hkv, D, S)
    ref_out = gpu.allocate((B, H, D), np.float32)
    na_out = gpu.allocate((B, H, D), np.float32)
    oracle = ops.gqa_decode(q, kc, vc, lens)
    for _ in range(2):
        gpu.memset(na_out, 0xFF)  # NaN pattern: every row must be rewritten
        gqa_decode(qd, kd, vd, ld, ref_out, max_len=S, workspace=ws)
        st = lib.tllm_gqa_decode_noalloc(qd.ptr, kd.ptr, vd.ptr, _lib.BF16, ld.ptr,
                                         na_out.ptr, B, H, Hkv, D, S, S, 0.0, None)
        _lib.check(st, "tllm_gqa_decode_noalloc")
        gpu.synchronize()
        a = ref_out.to_numpy()
        b = na_out.to_numpy()
        assert np.all(np.isfinite(b))
        np.testing.assert_allclose(b, a, atol=ATOL)
        np.testing.assert_allclose(b, oracle, atol=ATOL)


def test_noalloc_rejects_batches_over_its_limit():
    from triton_llm import _lib, gpu

    gpu._initialize()
    lib = _lib.load()
    # 65536 / 9 heads -> 7281 sequences fit; 7282 do not. The size check
    # happens before any pointer is touched, so null tensors are fine here.
    st = lib.tllm_gqa_decode_noalloc(None, None, None, _lib.BF16, None, None,
                                     7282, 9, 3, 64, 2048, 2048, 0.0, None)
    assert st == _lib.ERR_INVALID_ARG
    assert "65536" in _lib.last_error()


def _expected_splits(B, H, D, max_len, cap=8 << 20, rows=64, max_splits_cap=128):
    """Split count the decode planner picks for max_len keys (64-key tiles,
    ~3/8 of the tiles per chunk, 3..32 tiles), then the fewer, longer
    splits the allocation-free entry point needs to keep its partials
    inside its fixed region; returns (default, within the region)."""
    tiles = -(-max_len // rows)
    chunk = min(max(-(-3 * tiles // 8), 3), 32)
    chunk = max(chunk, -(-tiles // max_splits_cap)) * rows
    splits0 = -(-max_len // chunk)
    splits = splits0
    while splits > 1 and B * H * splits * (D + 2) * 4 > cap:
        chunk += rows
        splits = -(-max_len // chunk)
    return splits0, splits


@pytest.mark.parametrize("B,H,Hkv,D,S", [
    (192, 24, 8, 128, 8192),   # Llama-3.2-3B heads: 4 splits shrink to 3
    (2048, 9, 3, 64, 2048),    # SmolLM2 heads: 3 splits shrink to one
])
def test_noalloc_fewer_splits_when_partials_exceed_its_region(B, H, Hkv, D, S):
    """Batches whose split partials would not fit the fixed 8 MiB region run
    with fewer, longer splits (down to a single split): same results as the
    allocating entry point (which keeps the default split count) and the
    oracle, on two calls in a row."""
    from triton_llm import _lib, gpu
    from triton_llm.kernels import DecodeWorkspace, gqa_decode

    s0, s1 = _expected_splits(B, H, D, S)
    assert s1 < s0, "the case must exceed the region at the default split count"
    gpu._initialize()
    lib = _lib.load()
    rng = np.random.default_rng(11)
    lens = rng.integers(1, S + 1, B).astype(np.int32)
    lens[:2] = (S, S // 2 + 7)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    kd = gpu.allocate((B, Hkv, S, D), "bfloat16")
    vd = gpu.allocate((B, Hkv, S, D), "bfloat16")
    n = B * Hkv * S * D
    _lib.call("tllm_fill_random", kd.ptr, _lib.BF16, n, 21, 1.0, None)
    _lib.call("tllm_fill_random", vd.ptr, _lib.BF16, n, 22, 1.0, None)
    qd, ld = gpu.to_device(q), gpu.to_device(lens)
    ws = DecodeWorkspace(B, H, Hkv, D, S)
    ref_out = gpu.allocate((B, H, D), np.float32)
    na_out = gpu.allocate((B, H, D), np.float32)
    gqa_decode(qd, kd, vd, ld, ref_out, max_len=S, workspace=ws)
    a = ref_out.to_numpy()
    shp = (2, Hkv, S, D)
    kc = gpu.to_host(gpu.sub_view(kd, 0, shp))
    vc = gpu.to_host(gpu.sub_view(vd, 0, shp))
    want = ops.gqa_decode(q[:2], kc, vc, lens[:2])
    code = ctypes.c_int(-1)
    _lib.call("tllm_gqa_decode_noalloc_error", ctypes.byref(code), 1)
    for _ in range(2):
        gpu.memset(na_out, 0xFF)
        st = lib.tllm_gqa_decode_noalloc(qd.ptr, kd.ptr, vd.ptr, _lib.BF16, ld.ptr,
                                         na_out.ptr, B, H, Hkv, D, S, S, 0.0, None)
        _lib.check(st, "tllm_gqa_decode_noalloc")
        gpu.synchronize()
        b = na_out.to_numpy()
        assert np.all(np.isfinite(b))
        np.testing.assert_allclose(b, a, atol=ATOL)
        np.testing.assert_allclose(b[:2], want, atol=ATOL)
    _lib.call("tllm_gqa_decode_noalloc_error", ctypes.byref(code), 1)
    assert code.value == 0


def test_noalloc_error_word_reports_clamped_lengths():
    """A sequence longer than the caller's max_len bound is clamped on the
    device; the allocation-free call reports it in its own error word, which
    tllm_gqa_decode_noalloc_error reads and clears."""
    from triton_llm import _lib, gpu

    gpu._initialize()
    lib = _lib.load()
    B, H, Hkv, D, S = 4, 9, 3, 64, 2048
    lens, q, ks, vs = inputs.cfg2_inputs(batch=B, lo=1500, hi=2048)
    kd = gpu.to_device_bf16(inputs.pack_cache(ks, S))
    vd = gpu.to_device_bf16(inputs.pack_cache(vs, S))
    qd, ld = gpu.to_device(q), gpu.to_device(lens)
    out = gpu.allocate((B, H, D), np.float32)
    gpu.device_error(reset=True)
    code = ctypes.c_int(-1)
    _lib.call("tllm_gqa_decode_noalloc_error", ctypes.byref(code), 1)
    st = lib.tllm_gqa_decode_noalloc(qd.ptr, kd.ptr, vd.ptr, _lib.BF16, ld.ptr,
                                     out.ptr, B, H, Hkv, D, S, S, 0.0, None)
    _lib.check(st, "tllm_gqa_decode_noalloc")
    _lib.call("tllm_gqa_decode_noalloc_error", ctypes.byref(code), 0)
    assert code.value == 0
    # max_len 256 < every length (>= 1500): the kernel reads at most
    # 256 + one chunk keys of each sequence, all inside max_seq
    st = lib.tllm_gqa_decode_noalloc(qd.ptr, kd.ptr, vd.ptr, _lib.BF16, ld.ptr,
                                     out.ptr, B, H, Hkv, D, S, 256, 0.0, None)
    _lib.check(st, "tllm_gqa_decode_noalloc")
    _lib.call("tllm_gqa_decode_noalloc_error", ctypes.byref(code), 1)
    assert code.value & 2, f"clamp bit not set: {code.value}"
    _lib.call("tllm_gqa_decode_noalloc_error", ctypes.byref(code), 0)
    assert code.value == 0
    # the library-wide word is untouched by these calls
    assert gpu.device_error(reset=False) == 0
