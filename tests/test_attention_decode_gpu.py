"""Split-KV GQA decode kernel vs the oracle and the reference's goldens (GPU).

Tolerance: atol 1e-4, the reference's own GQA tolerance
(tests/test_attention_gqa.py:144). Inputs that are bf16 values are exactly
representable in both the fp32 and the bf16 cache, so the only difference to
the oracle is the order of fp32 accumulation.
"""

from __future__ import annotations

import numpy as np
import pytest

import inputs
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


def _upload_cache(gpu, arr, bf16):
    return gpu.to_device_bf16(arr) if bf16 else gpu.to_device(np.ascontiguousarray(arr, F32))


def _run_batched(gpu, q, kc, vc, lens, bf16, max_len=None, ws=None):
    from triton_llm.kernels import gqa_decode
    B, H, D = q.shape
    qd = gpu.to_device(np.ascontiguousarray(q, F32))
    kd = _upload_cache(gpu, kc, bf16)
    vd = _upload_cache(gpu, vc, bf16)
    ld = gpu.to_device(np.asarray(lens, np.int32))
    od = gpu.allocate((B, H, D), np.float32)
    gqa_decode(qd, kd, vd, ld, od, max_len=max_len, workspace=ws)
    gpu.synchronize()
    return od.to_numpy()


def test_flat_api_matches_reference_goldens(gpu, golden):
    """attention_gqa(seq_q=1) on the reference's own decode cases."""
    from triton_llm.kernels import attention_gqa
    g = golden("kernels")
    names = sorted({k.split("/")[1] for k in g if k.startswith("gqa/decode_")})
    assert names
    for n in names:
        nh, nkv, causal = (int(x) for x in g[f"gqa/{n}/meta"])
        o = attention_gqa(gpu.to_device(g[f"gqa/{n}/q"]), gpu.to_device(g[f"gqa/{n}/k"]),
                          gpu.to_device(g[f"gqa/{n}/v"]), nh, nkv, causal=bool(causal))
        gpu.synchronize()
        np.testing.assert_allclose(o.to_numpy(), g[f"gqa/{n}/out"], atol=ATOL,
                                   err_msg=n)


@pytest.mark.parametrize("bf16", [True, False])
def test_config2_full_batch(gpu, bf16):
    """64 ragged sequences, 9/3/64, lengths in [128, 2048]."""
    lens, q, ks, vs = inputs.cfg2_inputs()
    kc = inputs.pack_cache(ks, 2048)
    vc = inputs.pack_cache(vs, 2048)
    out = _run_batched(gpu, q, kc, vc, lens, bf16, max_len=2048)
    ref = ops.gqa_decode(q, kc, vc, lens)
    np.testing.assert_allclose(out, ref, atol=ATOL)


@pytest.mark.parametrize("H,Hkv,D", [(9, 3, 64), (24, 8, 128), (12, 12, 64),
                                     (32, 4, 128), (15, 3, 64), (16, 1, 64),
                                     (4, 2, 32), (8, 2, 256)])
@pytest.mark.parametrize("bf16", [True, False])
def test_ragged_edges(gpu, H, Hkv, D, bf16):
    """Lengths at tile and split edges, including an empty sequence."""
    rng = np.random.default_rng(H * 1000 + D)
    lens = np.array([0, 1, 31, 32, 33, 63, 64, 65, 127, 300, 1023, 1100], np.int32)
    S = 1152
    B = lens.size
    q = inputs.bf16_round(rng.standard_normal((B, H, D), dtype=F32))
    kc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    vc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    # rows past each length are poisoned: they must never be read into the sum
    for b, L in enumerate(lens):
        kc[b, :, L:] = np.nan
        vc[b, :, L:] = np.inf
    out = _run_batched(gpu, q, kc, vc, lens, bf16, max_len=int(lens.max()))
    ref = ops.gqa_decode(q, kc, vc, lens)
    assert np.all(np.isfinite(out))
    np.testing.assert_allclose(out, ref, atol=ATOL)
    assert np.all(out[0] == 0.0)


def test_long_context_many_splits(gpu):
    """Config-5 shard geometry (3 q heads on 1 KV head, d 128) at 32k keys."""
    rng = np.random.default_rng(5)
    B, H, Hkv, D, S = 2, 3, 1, 128, 32768
    lens = np.array([32768, 20001], np.int32)
    q = inputs.bf16_round(rng.standard_normal((B, H, D), dtype=F32))
    kc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    vc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    out = _run_batched(gpu, q, kc, vc, lens, True)
    ref = ops.gqa_decode(q, kc, vc, lens)
    np.testing.assert_allclose(out, ref, atol=ATOL)


def test_repeat_calls_are_deterministic(gpu):
    """Counters reset after each call: repeated calls give identical bits."""
    from triton_llm.kernels import gqa_decode, DecodeWorkspace
    lens, q, ks, vs = inputs.cfg2_inputs(batch=16)
    kd = gpu.to_device_bf16(inputs.pack_cache(ks, 2048))
    vd = gpu.to_device_bf16(inputs.pack_cache(vs, 2048))
    qd = gpu.to_device(q)
    ld = gpu.to_device(lens)
    ws = DecodeWorkspace(16, 9, 3, 64, 2048)
    outs = []
    for _ in range(3):
        od = gpu.allocate((16, 9, 64), np.float32)
        gqa_decode(qd, kd, vd, ld, od, max_len=2048, workspace=ws)
        outs.append(od.to_numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    assert np.all(ws.counters.to_numpy() == 0)


def test_rows_keys_hint_any_value(gpu):
    """tllm_gqa_rows_hint: the split sizes follow the caller's estimate of the
    keys read (a tiny hint: the shortest splits; the true sum: one wave; a
    huge hint: one split per row), and every plan matches the oracle and the
    call without a hint (16 ragged rows at Llama-3B head geometry, few
    enough row x KV-head pairs for the hint to apply)."""
    from triton_llm.kernels import DecodeWorkspace, gqa_rows
    rng = np.random.default_rng(21)
    B, H, Hkv, D, S = 16, 24, 8, 128, 4160
    lens = rng.integers(1024, 4096, B).astype(np.int32)
    q = inputs.bf16_round(rng.standard_normal((B, H, D), dtype=F32))
    kc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    vc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    for b, L in enumerate(lens):
        kc[b, :, L:] = np.nan
        vc[b, :, L:] = np.inf
    qd, kd, vd = gpu.to_device(q), gpu.to_device_bf16(kc), gpu.to_device_bf16(vc)
    ld = gpu.to_device(lens)
    ws = DecodeWorkspace(B, H, Hkv, D, S)
    ref = ops.gqa_decode(q, kc, vc, lens)
    outs = []
    for hint in (0, 1, int(lens.sum()), 10 ** 9):
        od = gpu.allocate((B, H, D), np.float32)
        gqa_rows(qd, kd, vd, None, ld, od, B, H, H * D, D, H * D, D, S,
                 workspace=ws, keys_hint=hint)
        outs.append(od.to_numpy())
        np.testing.assert_allclose(outs[-1], ref, atol=ATOL, err_msg=f"hint {hint}")
        np.testing.assert_allclose(outs[-1], outs[0], atol=ATOL, err_msg=f"hint {hint}")
    assert np.all(ws.counters.to_numpy() == 0)


def test_uniform_length_without_lens_array(gpu):
    rng = np.random.default_rng(3)
    B, H, Hkv, D, S = 3, 6, 2, 64, 500
    q = rng.standard_normal((B, H, D), dtype=F32)
    kc = rng.standard_normal((B, Hkv, S, D), dtype=F32)
    vc = rng.standard_normal((B, Hkv, S, D), dtype=F32)
    from triton_llm.kernels import gqa_decode
    od = gpu.allocate((B, H, D), np.float32)
    gqa_decode(gpu.to_device(q), gpu.to_device(kc), gpu.to_device(vc), None, od,
               max_len=S)
    ref = ops.gqa_decode(q, kc, vc, np.full(B, S))
    np.testing.assert_allclose(od.to_numpy(), ref, atol=ATOL)


@pytest.mark.parametrize("env", [{"TLLM_GQA_NO_MMA": "1"}, {}, {"TLLM_GQA_GROUPS": "1"},
                                 {"TLLM_GQA_GROUPS": "2"}])
def test_every_kernel_path(env):
    """Tensor-core and CUDA-core kernels each match the oracle on bf16; the
    tensor-core kernel with one and with two consumer groups at every head
    geometry (the default picks two at head_dim 64 with <= 8 heads per CTA)."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    script = Path(__file__).with_name("_gqa_paths_check.py")
    r = subprocess.run([sys.executable, str(script)], env={**os.environ, **env},
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
