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
