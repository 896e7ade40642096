"""Row, elementwise and projection kernels vs the reference's goldens and the
oracle (GPU).

Tolerances follow the reference's own kernel tests: 1e-5 for RMSNorm and
LayerNorm (tests/test_rms_norm.py, tests/test_layernorm.py), 1e-6 relative
for SwiGLU / add (exact up to expf), 1e-4 for RoPE and GEMM. The fused
projection (tllm_linear) is checked against an fp64 product of the weights
the device holds; bf16 weights are exact, the activations are split into a
bf16 head and residual, so the bound is 3e-5 of the row's sum |x| |w|.
KV append through the QKV epilogue is checked bit-exact against the oracle's
rotation of the same projection output. Temperature / top-k draws equal the
oracle's (itself pinned to the reference's _sample) unless the uniform lies
within 1e-6 of every cdf boundary between the two draws.
"""

from __future__ import annotations

import numpy as np
import pytest

import inputs
from oracle import ops

pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(scope="module")
def gpu():
    from triton_llm import gpu as g
    g._initialize()
    g.device_error(reset=True)
    yield g
    assert g.device_error(reset=True) == 0, "kernel reported a device error"


# ---------------------------------------------------------------- goldens --
def test_rmsnorm_golden(gpu, golden):
    from triton_llm.kernels import rms_norm
    g = golden("kernels")
    for key in sorted(k for k in g if k.startswith("rms/") and k.endswith("/x")):
        name = key.split("/")[1]
        x, w = g[f"rms/{name}/x"], g[f"rms/{name}/w"]
        o = gpu.allocate(x.shape, np.float32)
        rms_norm(gpu.to_device(x), gpu.to_device(w), o, 1e-5)
        np.testing.assert_allclose(o.to_numpy(), g[f"rms/{name}/out"], rtol=1e-5,
                                   atol=1e-5, err_msg=name)
    o = gpu.allocate((1, 1), np.float32)
    rms_norm(gpu.to_device(np.array([[3.0]], F32)), gpu.to_device(np.array([2.0], F32)),
             o, 1e-5)
    np.testing.assert_allclose(o.to_numpy(), g["rms/known/out"], rtol=1e-6)


def test_layernorm_golden(gpu, golden):
    from triton_llm.kernels import layer_norm
    g = golden("kernels")
    for name in ("3_768", "2_100"):
        out = layer_norm(g[f"ln/{name}/x"], g[f"ln/{name}/g"], g[f"ln/{name}/b"], 1e-5)
        np.testing.assert_allclose(out, g[f"ln/{name}/out"], rtol=1e-5, atol=1e-5)


def test_elementwise_golden(gpu, golden):
    from triton_llm.kernels import add, gelu, swiglu
    g = golden("kernels")
    x, y = g["swiglu/x"], g["swiglu/y"]
    s = swiglu(gpu.to_device(x), gpu.to_device(y)).to_numpy()
    np.testing.assert_allclose(s, g["swiglu/out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gelu(x), g["gelu/out"], rtol=1e-6, atol=1e-6)
    a = add(gpu.to_device(x), gpu.to_device(y)).to_numpy()
    np.testing.assert_array_equal(a, g["add/out"])


def test_embedding_golden(gpu, golden):
    from triton_llm.kernels import embedding
    g = golden("kernels")
    out = embedding(g["emb/ids"], g["emb/wte"], g["emb/wpe"], position_offset=9)
    np.testing.assert_array_equal(out, g["emb/out"])


def test_gemm_golden(gpu, golden):
    from triton_llm.kernels import gemm
    g = golden("kernels")
    for name in ("1_576_192", "3_64_100", "5_130_70"):
        a, b = g[f"gemm/{name}/a"], g[f"gemm/{name}/b"]
        o = gemm(gpu.to_device(a), gpu.to_device(b)).to_numpy()
        np.testing.assert_allclose(o, g[f"gemm/{name}/out"], rtol=1e-4, atol=1e-4,
                                   err_msg=name)


def test_rope_golden(gpu, golden):
    from triton_llm.kernels import apply_rope, precompute_cos_sin
    g = golden("kernels")
    c, s = precompute_cos_sin(256, 64, 100000.0)
    for key in [k for k in g if k.startswith("rope/apply/") and k.endswith("/x")]:
        name = key.split("/")[2]
        x = g[key]
        if name.endswith("_d128"):
            cc, ss = precompute_cos_sin(8192, 128, 500000.0)
            seq, off = 1, 8000
        else:
            cc, ss = c, s
            _, seq, off = (int(t) for t in name.split("_"))
        xd = gpu.to_device(x)
        apply_rope(xd, gpu.to_device(cc), gpu.to_device(ss), seq_len=seq,
                   position_offset=off)
        np.testing.assert_allclose(xd.to_numpy(), g[f"rope/apply/{name}/out"],
                                   rtol=1e-5, atol=1e-5, err_msg=name)


def test_softmax_and_argmax(gpu):
    from triton_llm import _lib
    from triton_llm.kernels import softmax
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((5, 49152)) * 4).astype(F32)
    np.testing.assert_allclose(softmax(x), ops.softmax(x), rtol=1e-5, atol=1e-9)
    # argmax: first maximal index wins, like np.argmax
    x[1, 100] = x[1, 7] = 1e3
    x[3, :] = 0.0
    xd = gpu.to_device(x)
    ids = gpu.zeros((5,), np.int32)
    pos = gpu.to_device(np.arange(5, dtype=np.int32))
    _lib.call("tllm_argmax", xd.ptr, 5, 49152, 49152, ids.ptr, pos.ptr, None)
    np.testing.assert_array_equal(ids.to_numpy(), np.argmax(x, axis=-1))
    np.testing.assert_array_equal(pos.to_numpy(), np.arange(5) + 1)


def _sample_dev(gpu, x, temperature, top_k, us, ld=None, pos=None):
    """tllm_sample over the rows of x (M, V) (row stride ld), uniforms us."""
    from triton_llm import _lib
    M, V = x.shape
    ld = ld or V
    xs = np.zeros((M, ld), F32)
    xs[:, :V] = x
    xd = gpu.to_device(xs)
    ud = gpu.to_device(np.asarray(us, np.float64).reshape(M))
    ids = gpu.zeros((M,), np.int32)
    _lib.call("tllm_sample", xd.ptr, M, V, ld, float(temperature), int(top_k),
              ud.ptr, ids.ptr, pos.ptr if pos is not None else None, None)
    return ids.to_numpy()


SAMPLE_BOUNDARY = 1e-6   # |cdf - u| inside which fp32 exp ulps may flip a draw


def _check_draw(got, x, T, k, u, label):
    """got must be the oracle's draw, unless u lies within SAMPLE_BOUNDARY of
    every cdf boundary between the two (the device's expf and summation
    order differ from NumPy's by ulps). Returns 1 for such a flip."""
    want = ops.sample(x, T, k, u)
    if got == want:
        return 0
    cdf = ops.sample_cdf(x, T, k)
    lo, hi = min(got, want), max(got, want)
    gap = float(np.max(np.abs(cdf[lo:hi] - u)))
    w = cdf[got] - (cdf[got - 1] if got else 0.0)
    assert gap < SAMPLE_BOUNDARY and w > 0, (
        f"{label}: drew {got}, oracle {want} (u={u!r}, cdf gap {gap:.3g}, "
        f"weight of {got} {w:.3g})")
    return 1


def test_sample_matches_reference_cases(gpu, golden):
    """Every reference _sample case (V 100..128256, T 0.3..1.5, top_k 0, 1,
    5, 50, 1000, V, V + 7): the device draws the reference's token with the
    uniform np.random.choice draws."""
    g = golden("sample")
    flips = 0
    for c, want in zip(inputs.SAMPLE_CASES, g["case_tokens"]):
        x = inputs.sample_logits(c)
        u = inputs.sample_uniform(c.rng)[0]
        got = int(_sample_dev(gpu, x[None], c.temperature, c.top_k, [u])[0])
        flip = _check_draw(got, x, c.temperature, c.top_k, u, str(c))
        assert got == int(want) or flip, (c, got, int(want))
        flips += flip
    print(f"sample cases: {len(inputs.SAMPLE_CASES) - flips}/"
          f"{len(inputs.SAMPLE_CASES)} identical to the reference")


@pytest.mark.parametrize("V,T,k,pad", [(49152, 1.0, 0, 0), (49152, 0.7, 50, 0),
                                       (128256, 0.7, 0, 64), (128256, 1.3, 1000, 64),
                                       (50257, 0.5, 7, 3)])
def test_sample_uniform_sweep_vs_oracle(gpu, V, T, k, pad):
    """256 rows of one logits vector with uniforms spread over [0, 1): each
    draw equals the oracle's (rows strided by V + pad)."""
    rng = np.random.default_rng(V + k)
    x = (rng.standard_normal(V) * 4).astype(F32)
    us = (np.arange(256) + rng.random(256)) / 256.0
    got = _sample_dev(gpu, np.repeat(x[None], 256, 0), T, k, us, ld=V + pad)
    flips = sum(_check_draw(int(gv), x, T, k, float(u), f"V={V} T={T} k={k}")
                for gv, u in zip(got, us))
    assert flips <= 1
    assert len(set(got.tolist())) >= min(k or 10, 5)   # the draws spread


def test_sample_edges(gpu):
    from triton_llm import _lib
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((4, 3000)) * 2).astype(F32)
    # top_k = 1 is the first argmax, whatever u is
    x[2, [17, 2500]] = 50.0
    got = _sample_dev(gpu, x, 0.9, 1, [0.0, 0.5, 0.99, 0.999999])
    np.testing.assert_array_equal(got, np.argmax(x, axis=-1))
    # equal logits at the threshold keep the lowest indices
    y = np.zeros((64, 4096), F32)
    y[:, [2, 5, 7, 4000]] = 1.0
    us = np.linspace(0.0, 0.999, 64)
    got = _sample_dev(gpu, y, 1.0, 2, us)
    assert set(got.tolist()) == {2, 5}
    for gv, u in zip(got, us):
        _check_draw(int(gv), y[0], 1.0, 2, float(u), "ties")
    # more equal logits at the threshold than the shared buffer holds: the
    # remaining digits and the index cut are selected over the whole row
    z = np.zeros((64, 49152), F32)
    z[:, ::7] = 1.0
    us = np.linspace(0.0, 0.999, 64)
    got = _sample_dev(gpu, z, 1.0, 10000, us)
    for gv, u in zip(got, us):
        _check_draw(int(gv), z[0], 1.0, 10000, float(u), "wide tie")
    assert np.any(got % 7 != 0)   # kept zeros (the lowest indices) are drawn
    # top_k >= V is top_k = 0; pos advances by one
    pos = gpu.to_device(np.array([3, 9], np.int32))
    a = _sample_dev(gpu, x[:2], 1.1, 3000, [0.25, 0.75], pos=pos)
    b = _sample_dev(gpu, x[:2], 1.1, 0, [0.25, 0.75])
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(pos.to_numpy(), [4, 10])
    # u = 0 draws the first index, u just below 1 the last
    got = _sample_dev(gpu, x[:2], 1.0, 0, [0.0, np.nextafter(1.0, 0.0)])
    np.testing.assert_array_equal(got, [0, 2999])
    # M = 0 is a no-op; a greedy temperature and a negative top_k are refused
    _lib.call("tllm_sample", None, 0, 10, 10, 1.0, 0, None, None, None, None)
    xd, ud, ids = gpu.to_device(x), gpu.zeros((4,), np.float64), gpu.zeros((4,), np.int32)
    with pytest.raises(ValueError):
        _lib.call("tllm_sample", xd.ptr, 4, 3000, 3000, 1e-7, 0, ud.ptr, ids.ptr, None, None)
    with pytest.raises(ValueError):
        _lib.call("tllm_sample", xd.ptr, 4, 3000, 3000, 1.0, -1, ud.ptr, ids.ptr, None, None)


def test_sample_time_at_config4_rows(gpu):
    """64 rows of the Llama vocabulary (config 4's batch) in one launch: the
    draw costs a small fraction of a decode step (printed)."""
    from triton_llm import _lib
    rng = np.random.default_rng(4)
    xd = gpu.to_device((rng.standard_normal((64, 128256)) * 3).astype(F32))
    ud = gpu.to_device(rng.random(64))
    ids = gpu.zeros((64,), np.int32)
    for rows, k in ((64, 0), (64, 50), (64, 1000), (1, 0), (1, 50)):
        for _ in range(3):
            _lib.call("tllm_sample", xd.ptr, rows, 128256, 128256, 0.8, k, ud.ptr,
                      ids.ptr, None, None)
        e0, e1 = gpu.Event(), gpu.Event()
        e0.record()
        for _ in range(20):
            _lib.call("tllm_sample", xd.ptr, rows, 128256, 128256, 0.8, k, ud.ptr,
                      ids.ptr, None, None)
        e1.record()
        gpu.synchronize()
        us = e0.elapsed_ms(e1) * 1e3 / 20
        print(f"tllm_sample {rows} x 128256 top_k={k}: {us:.1f} us "
              f"({rows * 128256 * 4 / us / 1e3:.0f} GB/s of logits)")
        assert us < 1000.0


def test_fill_random_matches_host_formula(gpu):
    """The device N(0, std) fill is reproducible on the host (splitmix64
    hash, Irwin-Hall sum of four 16-bit fields)."""
    from triton_llm import _lib
    n, seed, std = 4099, 77, 0.02
    t = gpu.allocate((n,), np.float32)
    _lib.call("tllm_fill_random", t.ptr, _lib.F32, n, seed, float(std), None)
    got = t.to_numpy()

    def mix64(z):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))

    with np.errstate(over="ignore"):
        h = mix64(np.uint64(seed) ^ mix64(np.arange(n, dtype=np.uint64)))
    s = sum(((h >> np.uint64(16 * i)) & np.uint64(0xFFFF)).astype(np.int64)
            for i in range(4))
    scale = F32(std) / (F32(65536.0) * F32(0.57735026918962576))
    ref = (s - 131070).astype(F32) * scale
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-9)
    assert abs(got.std() - std) < 0.05 * std


# ------------------------------------------------------- fused projection --
def _linear_case(gpu, M, N, K, bf16, seed=0):
    from triton_llm.kernels.linear import Linear
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K), dtype=F32) * 0.05).astype(F32)
    x = rng.standard_normal((M, K), dtype=F32)
    lin = Linear(w, "bfloat16" if bf16 else "float32")
    wd = ops.bf16_round(w) if bf16 else w
    ref = x.astype(np.float64) @ wd.astype(np.float64).T
    bound = np.abs(x).astype(np.float64) @ np.abs(wd).astype(np.float64).T
    return lin, x, wd, ref, bound


def _close(out, ref, bound, rel=3e-5, msg=""):
    err = np.abs(out.astype(np.float64) - ref)
    lim = rel * bound + 1e-6
    bad = err > lim
    assert not bad.any(), f"{msg}: {bad.sum()} outside bound, worst {(err / lim).max():.2f}x"


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 17, 33, 64, 100, 130])
def test_linear_store_bias(gpu, M, bf16):
    from triton_llm.kernels.linear import LinearWorkspace, linear
    N, K = 576, 576
    lin, x, wd, ref, bound = _linear_case(gpu, M, N, K, bf16, seed=M)
    b = np.linspace(-1, 1, N).astype(F32)
    from triton_llm import gpu as g
    lin.b = g.to_device(b)
    out = gpu.allocate((M, N), np.float32)
    linear(gpu.to_device(x), lin, out_dev=out, ws=LinearWorkspace([(M, N, K)]), M=M)
    _close(out.to_numpy(), ref + b, bound, msg=f"M={M}")


@pytest.mark.parametrize("planes", [1, 2])
@pytest.mark.parametrize("M", [1, 7, 16, 32])
@pytest.mark.parametrize("op", ["store", "resid", "gelu", "swiglu"])
def test_linear_skinny_matches_tensor_core_kernel(gpu, monkeypatch, op, M, planes):
    """Batches up to 32 rows take the mma.sync skinny kernel; it gives what
    the tcgen05 kernel gives on the same operands (both sum in fp32, in a
    different order)."""
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear, swiglu_rows
    rng = np.random.default_rng(60 + M)
    N, K = (1536, 576) if op == "swiglu" else (576, 1536)
    w = rng.standard_normal((N, K), dtype=F32) * 0.05
    if op == "swiglu":
        w = swiglu_rows(w[:N // 2], w[N // 2:])
    lin = Linear(w.astype(F32), "bfloat16", np.linspace(-1, 1, N).astype(F32)
                 if op in ("store", "gelu") else None)
    x = gpu.to_device_split(rng.standard_normal((M, K), dtype=F32), planes=planes)
    h0 = rng.standard_normal((M, N), dtype=F32)
    code = {"store": _lib.EPI_STORE, "resid": _lib.EPI_RESID, "gelu": _lib.EPI_GELU,
            "swiglu": _lib.EPI_SWIGLU}[op]
    ws = LinearWorkspace([(M, N, K)])
    outs = []
    for max_m in ("32", "0"):   # skinny kernel, then the tcgen05 kernel
        monkeypatch.setenv("TLLM_SKINNY_MAX_M", max_m)
        out = gpu.to_device(h0) if op == "resid" else gpu.allocate(
            (M, N // 2 if op == "swiglu" else N), np.float32)
        linear(x, lin, out_dev=out, op=code, resid_dev=out if op == "resid" else None,
               ws=ws, M=M)
        outs.append(out.to_numpy())
    scale = np.abs(outs[1]).max()
    np.testing.assert_allclose(outs[0], outs[1], rtol=1e-4, atol=1e-5 * scale)


@pytest.mark.parametrize("bf16", [True, False])
def test_linear_split_k_deterministic(gpu, bf16):
    """Few weight tiles and long K: the kernel splits K across CTAs and the
    last CTA sums the splits in a fixed order -> bitwise repeatable."""
    from triton_llm.kernels.linear import LinearWorkspace, linear
    M, N, K = 4, 256, 8192
    lin, x, wd, ref, bound = _linear_case(gpu, M, N, K, bf16, seed=11)
    ws = LinearWorkspace([(M, N, K)])
    xd = gpu.to_device(x)
    outs = []
    for _ in range(3):
        out = gpu.allocate((M, N), np.float32)
        linear(xd, lin, out_dev=out, ws=ws, M=M)
        outs.append(out.to_numpy())
    _close(outs[0], ref, bound, msg="split-K")
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
    # the counters are left at zero for the next call / graph replay
    assert not ws.counters.to_numpy().any()


@pytest.mark.parametrize("bf16", [True, False])
def test_linear_residual_in_place(gpu, bf16):
    from triton_llm import _lib
    from triton_llm.kernels.linear import LinearWorkspace, linear
    M, N, K = 5, 576, 1536
    lin, x, wd, ref, bound = _linear_case(gpu, M, N, K, bf16, seed=5)
    h = np.random.default_rng(6).standard_normal((M, N), dtype=F32)
    hd = gpu.to_device(h)
    linear(gpu.to_device(x), lin, out_dev=hd, op=_lib.EPI_RESID, resid_dev=hd,
           ws=LinearWorkspace([(M, N, K)]), M=M)
    _close(hd.to_numpy(), ref + h, bound, msg="resid")


@pytest.mark.parametrize("bf16", [True, False])
def test_linear_gelu(gpu, bf16):
    from triton_llm import _lib
    from triton_llm.kernels.linear import LinearWorkspace, linear
    M, N, K = 7, 3072, 768
    lin, x, wd, ref, bound = _linear_case(gpu, M, N, K, bf16, seed=7)
    out = gpu.allocate((M, N), np.float32)
    linear(gpu.to_device(x), lin, out_dev=out, op=_lib.EPI_GELU,
           ws=LinearWorkspace([(M, N, K)]), M=M)
    # gelu' <= 1.13: the product bound carries over
    np.testing.assert_allclose(out.to_numpy(), ops.gelu(ref.astype(F32)),
                               atol=1.2 * 3e-5 * bound.max() + 1e-6)


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("M", [1, 64])
def test_linear_swiglu(gpu, M, bf16):
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear, swiglu_rows
    F, K = 1536, 576
    rng = np.random.default_rng(M)
    wg = (rng.standard_normal((F, K), dtype=F32) * 0.05).astype(F32)
    wu = (rng.standard_normal((F, K), dtype=F32) * 0.05).astype(F32)
    x = rng.standard_normal((M, K), dtype=F32)
    dt = "bfloat16" if bf16 else "float32"
    lin = Linear(swiglu_rows(wg, wu), dt)
    rd = ops.bf16_round if bf16 else (lambda a: a)
    gref = x.astype(np.float64) @ rd(wg).astype(np.float64).T
    uref = x.astype(np.float64) @ rd(wu).astype(np.float64).T
    out = gpu.allocate((M, F), np.float32)
    linear(gpu.to_device(x), lin, out_dev=out, op=_lib.EPI_SWIGLU,
           ws=LinearWorkspace([(M, 2 * F, K)]), M=M)
    ref = ops.swiglu(gref.astype(F32), uref.astype(F32))
    np.testing.assert_allclose(out.to_numpy(), ref, rtol=2e-4, atol=2e-4)


def test_linear_rejects_bad_shapes(gpu):
    from triton_llm.kernels.linear import Linear, linear
    with pytest.raises(ValueError):     # bf16 weights need K % 64 == 0
        Linear(np.zeros((16, 96), F32), "bfloat16")
    lin = Linear(np.zeros((16, 64), F32), "bfloat16")
    with pytest.raises(ValueError):
        linear(gpu.allocate((1, 32), np.float32), lin, out_dev=gpu.allocate((1, 16), np.float32))


@pytest.mark.parametrize("kv_bf16", [True, False])
@pytest.mark.parametrize("w_bf16", [True, False])
@pytest.mark.parametrize("H,Hkv,D", [(9, 3, 64), (24, 8, 128), (4, 2, 16)])
def test_qkv_rope_append_bit_exact(gpu, H, Hkv, D, w_bf16, kv_bf16):
    """QKV epilogue: q rotated into q_out, k rotated and v appended at
    (seq, kv_head, pos) of the cache, lens_out[seq] = pos + 1 -- bit-exact
    against the oracle's RoPE applied to the same projection (EPI_STORE of
    the same weights runs the same reduction order)."""
    from triton_llm import _lib
    from triton_llm.kernels.linear import (Linear, LinearWorkspace, head_row_order,
                                           linear, qkv_rows)
    n = H * D
    K = 576 if D != 16 else 64
    rows = (H + 2 * Hkv) * D
    rng = np.random.default_rng(H * 1000 + D)
    wq = (rng.standard_normal((H * D, K), dtype=F32) * 0.05).astype(F32)
    wk = (rng.standard_normal((Hkv * D, K), dtype=F32) * 0.05).astype(F32)
    wv = (rng.standard_normal((Hkv * D, K), dtype=F32) * 0.05).astype(F32)
    B, S, M = 3, 40, 5
    x = rng.standard_normal((M, K), dtype=F32)
    row_seq = np.array([0, 2, 2, 1, 0], np.int32)
    row_pos = np.array([0, 17, 18, 39, 1], np.int32)
    cos, sin = ops.precompute_cos_sin(64, D, 100000.0)
    dt = "bfloat16" if w_bf16 else "float32"
    wperm, _ = qkv_rows(wq, wk, wv, D)
    lin = Linear(wperm, dt)
    ws = LinearWorkspace([(M, rows, K)])
    xd = gpu.to_device(x)
    # plain projection with the same weights and shape -> same sums
    plain = gpu.allocate((M, rows), np.float32)
    linear(xd, lin, out_dev=plain, ws=ws, M=M)
    y = plain.to_numpy()
    inv = np.argsort(np.concatenate([h * D + head_row_order(D)
                                     for h in range(H + 2 * Hkv)]))
    y = y[:, inv]                                  # back to natural head order
    q, k, v = y[:, :n], y[:, n:n + Hkv * D], y[:, n + Hkv * D:]
    kvdt = "bfloat16" if kv_bf16 else np.float32
    kc = gpu.zeros((B, Hkv, S, D), kvdt)
    vc = gpu.zeros((B, Hkv, S, D), kvdt)
    q_out = gpu.allocate((M, H, D), np.float32)
    lens = gpu.zeros((B,), np.int32)
    linear(xd, lin, op=_lib.EPI_QKV, ws=ws, M=M, qkv=dict(
        cos=gpu.to_device(cos), sin=gpu.to_device(sin), row_seq=gpu.to_device(row_seq),
        row_pos=gpu.to_device(row_pos), q_out=q_out, k_cache=kc, v_cache=vc,
        n_head=H, n_kv_head=Hkv, head_dim=D, lens_out=lens))
    qr = ops.rope_positions(q.reshape(M * H, D), cos, sin,
                            np.repeat(row_pos, H)).reshape(M, H, D)
    kr = ops.rope_positions(k.reshape(M * Hkv, D), cos, sin,
                            np.repeat(row_pos, Hkv)).reshape(M, Hkv, D)
    np.testing.assert_array_equal(q_out.to_numpy(), qr)
    kexp = np.zeros((B, Hkv, S, D), F32)
    vexp = np.zeros((B, Hkv, S, D), F32)
    for m in range(M):
        kexp[row_seq[m], :, row_pos[m]] = kr[m]
        vexp[row_seq[m], :, row_pos[m]] = v[m].reshape(Hkv, D)
    st = ops.bf16_round if kv_bf16 else (lambda a: a)
    np.testing.assert_array_equal(gpu.to_host(kc), st(kexp))
    np.testing.assert_array_equal(gpu.to_host(vc), st(vexp))
    # every row writes lens_out[seq] = pos + 1; rows of one sequence race, so
    # only sequences written by one row (or ordered by position) are pinned
    got = lens.to_numpy()
    assert got[1] == 40
    assert got[0] in (1, 2) and got[2] in (18, 19)


def test_qkv_rejects_out_of_range_position(gpu):
    """A position outside the cache is not written; the kernel flags it."""
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear, qkv_rows
    H, Hkv, D, K = 2, 1, 64, 64
    w = np.ones(((H + 2 * Hkv) * D, K), F32) * 0.01
    lin = Linear(w, "bfloat16")
    kc = gpu.zeros((1, Hkv, 8, D), "bfloat16")
    vc = gpu.zeros((1, Hkv, 8, D), "bfloat16")
    gpu.device_error(reset=True)
    linear(gpu.to_device(np.ones((1, K), F32)), lin, op=_lib.EPI_QKV,
           ws=LinearWorkspace([(1, w.shape[0], K)]), M=1, qkv=dict(
               row_seq=gpu.zeros((1,), np.int32),
               row_pos=gpu.to_device(np.array([8], np.int32)),
               q_out=gpu.allocate((1, H, D), np.float32), k_cache=kc, v_cache=vc,
               n_head=H, n_kv_head=Hkv, head_dim=D))
    gpu.synchronize()
    assert gpu.device_error(reset=True) & 2
    assert not gpu.to_host(kc).any() and not gpu.to_host(vc).any()


# ----------------------------------------------------- prefill attention --
def test_prefill_flat_matches_reference_goldens(gpu, golden):
    """attention_gqa(seq_q > 1, causal) on the reference's prefill cases."""
    from triton_llm.kernels import attention_gqa
    g = golden("kernels")
    names = sorted({k.split("/")[1] for k in g
                    if k.startswith("gqa/prefill_") or k.startswith("gqa/causal_")})
    assert len(names) >= 6
    for n in names:
        nh, nkv, causal = (int(x) for x in g[f"gqa/{n}/meta"])
        o = attention_gqa(gpu.to_device(g[f"gqa/{n}/q"]), gpu.to_device(g[f"gqa/{n}/k"]),
                          gpu.to_device(g[f"gqa/{n}/v"]), nh, nkv, causal=bool(causal))
        gpu.synchronize()
        np.testing.assert_allclose(o.to_numpy(), g[f"gqa/{n}/out"], atol=1e-4,
                                   err_msg=n)


@pytest.mark.parametrize("bf16", [True, False])
def test_gqa_rows_ragged_prefill(gpu, bf16):
    """Row API: rows of three sequences, each attending its own prefix."""
    from triton_llm.kernels import gqa_rows
    H, Hkv, D, S = 9, 3, 64, 300
    rng = np.random.default_rng(9)
    kc = ops.bf16_round(rng.standard_normal((3, Hkv, S, D), dtype=F32))
    vc = ops.bf16_round(rng.standard_normal((3, Hkv, S, D), dtype=F32))
    row_seq = np.array([0, 0, 1, 2, 2, 2, 1], np.int32)
    row_len = np.array([1, 2, 300, 64, 65, 129, 0], np.int32)
    R = len(row_seq)
    q = rng.standard_normal((R, H, D), dtype=F32)
    up = gpu.to_device_bf16 if bf16 else gpu.to_device
    out = gpu.allocate((R, H * D), np.float32)
    gqa_rows(gpu.to_device(q), up(kc), up(vc), gpu.to_device(row_seq),
             gpu.to_device(row_len), out, R, H, H * D, D, H * D, D, S)
    got = out.to_numpy().reshape(R, H, D)
    ref = ops.gqa_decode(q, kc[row_seq], vc[row_seq], row_len)
    np.testing.assert_allclose(got, ref, atol=1e-4)


# ------------------------------------------------ split operand format --
def test_split_conversion_bit_exact(gpu):
    """tllm_split_bf16: plane 0 = bf16(x), plane 1 = bf16(x - hi), rows
    beyond `rows` untouched."""
    from triton_llm.kernels.linear import to_split
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((7, 320)) * 10).astype(F32)
    x[0, :4] = [0.0, -0.0, 1e-30, 3e38]
    xs = gpu.split_empty(9, 320)
    gpu.memset(xs, 0)
    to_split(gpu.to_device(x), out=xs)
    planes = xs.to_numpy()
    hi, lo = gpu.split_host(x)
    np.testing.assert_array_equal(planes[0, :7], hi)
    np.testing.assert_array_equal(planes[1, :7], lo)
    assert not planes[:, 7:].any()
    rel = np.abs(gpu.split_to_host(xs, 7) - x) / np.maximum(np.abs(x), 1e-30)
    assert rel.max() < 2 ** -16


@pytest.mark.parametrize("planes", [2, 1])
@pytest.mark.parametrize("norm", ["rms", "ln"])
def test_norm_split_output_equals_split_of_fp32(gpu, norm, planes):
    from triton_llm.kernels.rms_norm import rms_norm_rows
    from triton_llm.kernels.layernorm import layer_norm_dev
    rng = np.random.default_rng(2)
    M, N = 5, 576
    x = rng.standard_normal((M, N), dtype=F32)
    w = rng.standard_normal(N, dtype=F32)
    b = rng.standard_normal(N, dtype=F32)
    xd, wd, bd = gpu.to_device(x), gpu.to_device(w), gpu.to_device(b)
    f = gpu.allocate((M, N), np.float32)
    sp = gpu.act_empty(8, N, planes)
    if norm == "rms":
        rms_norm_rows(xd, wd, f, M)
        rms_norm_rows(xd, wd, sp, M)
    else:
        layer_norm_dev(xd, wd, bd, f, M=M)
        layer_norm_dev(xd, wd, bd, sp, M=M)
    hi, lo = gpu.split_host(f.to_numpy())
    got = sp.to_numpy()
    np.testing.assert_array_equal(got[0, :M], hi)
    if planes == 2:
        np.testing.assert_array_equal(got[1, :M], lo)


def test_linear_split_output_equals_split_of_fp32(gpu):
    """SwiGLU epilogue writing the operand format of the next projection."""
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear, swiglu_rows
    rng = np.random.default_rng(4)
    F, K, M = 256, 576, 6
    lin = Linear(swiglu_rows(rng.standard_normal((F, K), dtype=F32) * 0.05,
                             rng.standard_normal((F, K), dtype=F32) * 0.05), "bfloat16")
    xs = gpu.to_device_split(rng.standard_normal((M, K), dtype=F32), plane_rows=16)
    ws = LinearWorkspace([(M, 2 * F, K)])
    f = gpu.allocate((M, F), np.float32)
    sp = gpu.split_empty(16, F)
    linear(xs, lin, out_dev=f, op=_lib.EPI_SWIGLU, ws=ws, M=M)
    linear(xs, lin, out_dev=sp, op=_lib.EPI_SWIGLU, ws=ws, M=M)
    hi, lo = gpu.split_host(f.to_numpy())
    planes = sp.to_numpy()
    np.testing.assert_array_equal(planes[0, :M], hi)
    np.testing.assert_array_equal(planes[1, :M], lo)


@pytest.mark.parametrize("planes", [2, 1])
@pytest.mark.parametrize("M", [1, 16, 17, 64, 65, 200, 300, 600])
def test_linear_tile_shapes(gpu, M, planes):
    """Every activation tile width (16..256 columns), multiple row tiles,
    N not a multiple of the 128-row weight tile; hi + lo activations
    (near fp32) and bf16 activations (checked against the bf16-rounded
    input, exact products, fp32 sums)."""
    from triton_llm.kernels.linear import LinearWorkspace, linear
    N, K = 1000, 1024
    lin, x, wd, ref, bound = _linear_case(gpu, M, N, K, True, seed=100 + M)
    xs = gpu.to_device_split(x, planes=planes)
    if planes == 1:
        xr = ops.bf16_round(x).astype(np.float64)
        ref = xr @ wd.astype(np.float64).T
    out = gpu.allocate((M, N), np.float32)
    linear(xs, lin, out_dev=out, ws=LinearWorkspace([(M, N, K)]), M=M)
    _close(out.to_numpy(), ref, bound, rel=2e-6 if planes == 1 else 3e-5,
           msg=f"M={M} planes={planes}")


@pytest.mark.parametrize("planes", [2, 1])
def test_attention_split_output(gpu, planes):
    """gqa_rows writing the operand format of the o projection."""
    from triton_llm.kernels import gqa_rows
    H, Hkv, D, S, R = 24, 8, 128, 512, 5
    rng = np.random.default_rng(8)
    kc = ops.bf16_round(rng.standard_normal((R, Hkv, S, D), dtype=F32))
    vc = ops.bf16_round(rng.standard_normal((R, Hkv, S, D), dtype=F32))
    lens = np.array([1, 100, 512, 64, 300], np.int32)
    q = rng.standard_normal((R, H, D), dtype=F32)
    seq = np.arange(R, dtype=np.int32)
    args = (gpu.to_device(q), gpu.to_device_bf16(kc), gpu.to_device_bf16(vc),
            gpu.to_device(seq), gpu.to_device(lens))
    f = gpu.allocate((R, H * D), np.float32)
    sp = gpu.act_empty(8, H * D, planes)
    gqa_rows(*args, f, R, H, H * D, D, H * D, D, S)
    gqa_rows(*args, sp, R, H, H * D, D, H * D, D, S)
    hi, lo = gpu.split_host(f.to_numpy())
    got = sp.to_numpy()
    np.testing.assert_array_equal(got[0, :R], hi)
    if planes == 2:
        np.testing.assert_array_equal(got[1, :R], lo)


def test_first_call_inside_graph_capture(gpu):
    """A kernel entry point whose per-device state has not been created yet
    can be captured: the capture call creates it first."""
    import subprocess
    import sys
    code = (
        "import sys, numpy as np; sys.path.insert(0, 'triton-llm_b200');"
        "from triton_llm import gpu, _lib;"
        "from triton_llm.kernels.linear import Linear, linear;"
        "gpu._initialize();"
        "lin = Linear(np.ones((128, 64), np.float32) * 0.5, 'bfloat16');"
        "x = gpu.to_device_split(np.ones((2, 64), np.float32));"
        "out = gpu.allocate((2, 128), np.float32);"
        "g = gpu.Graph()\n"
        "with g:\n"
        "    linear(x, lin, out_dev=out, M=2)\n"
        "g.launch(); gpu.device_synchronize();"
        "assert np.allclose(out.to_numpy(), 32.0), out.to_numpy()[0, :4];"
        "print('ok')")
    from pathlib import Path
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       cwd=str(Path(__file__).resolve().parent.parent), timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


# ------------------------------------------------- fused peer all-reduce --
def _peer_group_1(rows, cols):
    """A one-rank peer group (the scatter writes this GPU's own slots)."""
    from triton_llm import gpu
    from triton_llm.tp import PeerGroup, TPGroup
    return PeerGroup(TPGroup(0, 1, gpu.current_device()), rows, cols)


@pytest.mark.parametrize("planes", [2, 1])
def test_scatter_then_rmsnorm_p2p_equals_store_then_rmsnorm_add(gpu, monkeypatch, planes):
    """SCATTER + tllm_rmsnorm_p2p on a one-rank group computes what STORE +
    tllm_rmsnorm_add computes, over several calls (both slot parities) and
    inside a replayed CUDA graph. SCATTER runs on the tcgen05 kernel, so the
    STORE side is held there too (bitwise comparison of the reduction)."""
    monkeypatch.setenv("TLLM_SKINNY_MAX_M", "0")
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear
    from triton_llm.kernels.rms_norm import rms_norm_add_rows, rms_norm_p2p_rows
    M, N, K = 5, 576, 1536
    rng = np.random.default_rng(31)
    lin = Linear((rng.standard_normal((N, K), dtype=F32) * 0.05).astype(F32), "bfloat16")
    wn = gpu.to_device(rng.standard_normal(N, dtype=F32))
    ws = LinearWorkspace([(M, N, K)])
    peer = _peer_group_1(8, N)
    h0 = rng.standard_normal((M, N), dtype=F32)
    h_ref, h_p2p = gpu.to_device(h0), gpu.to_device(h0)
    part = gpu.allocate((M, N), np.float32)
    y_ref, y_p2p = gpu.act_empty(M, N, planes), gpu.act_empty(M, N, planes)
    x = gpu.act_empty(M, K, planes)

    def check(tag):
        assert np.array_equal(h_p2p.to_numpy(), h_ref.to_numpy()), tag
        a, b = gpu.split_to_host(y_p2p), gpu.split_to_host(y_ref)
        np.testing.assert_allclose(a, b, rtol=2e-6, atol=1e-6, err_msg=tag)

    xs = [rng.standard_normal((M, K), dtype=F32) for _ in range(3)]
    for it, xv in enumerate(xs):
        gpu.copy_d2d(x, gpu.to_device_split(xv, planes=planes))
        linear(x, lin, out_dev=part, op=_lib.EPI_STORE, ws=ws, M=M)
        rms_norm_add_rows(h_ref, part, wn, y_ref, M)
        linear(x, lin, op=_lib.EPI_SCATTER, ws=ws, M=M, p2p=peer)
        rms_norm_p2p_rows(h_p2p, peer, wn, y_p2p, M)
        gpu.device_synchronize()
        check(f"call {it}")
    g = gpu.Graph()
    with g:
        linear(x, lin, op=_lib.EPI_SCATTER, ws=ws, M=M, p2p=peer)
        rms_norm_p2p_rows(h_p2p, peer, wn, y_p2p, M)
    for it in range(3):
        linear(x, lin, out_dev=part, op=_lib.EPI_STORE, ws=ws, M=M)
        rms_norm_add_rows(h_ref, part, wn, y_ref, M)
        g.launch()
        gpu.device_synchronize()
        check(f"replay {it}")
    del g
    peer.close()


def test_scatter_rejects_bad_arguments(gpu):
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear
    from triton_llm.kernels.rms_norm import rms_norm_p2p_rows
    N, K = 256, 128
    rng = np.random.default_rng(3)
    w = rng.standard_normal((N, K), dtype=F32)
    peer = _peer_group_1(4, N)
    x = gpu.act_empty(8, K, 2)
    ws = LinearWorkspace([(8, N, K)])
    with pytest.raises(ValueError):      # more rows than the slots hold
        linear(x, Linear(w, "bfloat16"), op=_lib.EPI_SCATTER, ws=ws, M=5, p2p=peer)
    with pytest.raises(ValueError):      # fp32 weights
        linear(gpu.to_device(np.zeros((4, K), F32)), Linear(w, "float32"),
               op=_lib.EPI_SCATTER, ws=ws, M=4, p2p=peer)
    with pytest.raises(ValueError):      # no group
        linear(x, Linear(w, "bfloat16"), op=_lib.EPI_SCATTER, ws=ws, M=4)
    with pytest.raises(ValueError):      # wider rows than the slots
        rms_norm_p2p_rows(gpu.allocate((4, 2 * N), np.float32), peer,
                          gpu.allocate((2 * N,), np.float32),
                          gpu.allocate((4, 2 * N), np.float32), 4)
    peer.close()


# ----------------------------------------------------- fused decode MLP block --
def _close_mlp(got, want, msg):
    # both paths sum in fp32 but in different orders (split-K pieces, the
    # norm's sum of squares) and round x and act to bf16 afterwards, so a
    # few elements land one bf16 step apart before the down projection;
    # every element stays within 5e-3 and the mean difference near zero
    np.testing.assert_allclose(got, want, rtol=5e-3, atol=5e-3, err_msg=msg)
    assert float(np.abs(got - want).mean()) < 2e-5, msg

@pytest.mark.parametrize("M,hidden,ffn", [(1, 1024, 2816), (8, 1024, 2816),
                                          (33, 1024, 2816), (64, 1024, 2816),
                                          (8, 256, 9600)])
def test_mlp_block_matches_the_four_launches(gpu, M, hidden, ffn):
    """tllm_mlp (o + residual, RMSNorm, gate/up + SwiGLU, down + residual in
    one launch) against the same layer as four launches, on two calls in a
    row and in a replayed CUDA graph (its counters survive between calls).
    The last shape has more gate/up tiles than SMs (whole tiles in turn)."""
    from triton_llm import _lib
    from triton_llm.kernels.linear import Linear, LinearWorkspace, linear, swiglu_rows
    from triton_llm.kernels.mlp import MlpWorkspace, mlp_block
    from triton_llm.kernels.rms_norm import rms_norm_rows
    attn_dim, eps = hidden, 1e-5
    rng = np.random.default_rng(40 + M)
    w = lambda n, k: (rng.standard_normal((n, k), dtype=F32) * 0.03).astype(F32)  # noqa: E731
    wo = Linear(w(hidden, attn_dim), "bfloat16")
    wgu = Linear(swiglu_rows(w(ffn, hidden), w(ffn, hidden)), "bfloat16")
    wd = Linear(w(hidden, ffn), "bfloat16")
    ln = gpu.to_device((1.0 + 0.1 * rng.standard_normal(hidden)).astype(F32))
    attn = gpu.to_device_split(rng.standard_normal((M, attn_dim), dtype=F32), planes=1)
    h0 = rng.standard_normal((M, hidden), dtype=F32)
    lws = LinearWorkspace([(M, hidden, attn_dim), (M, 2 * ffn, hidden), (M, hidden, ffn)])
    mws = MlpWorkspace(M, attn_dim, hidden, ffn)

    def four(h):
        x = gpu.act_empty(M, hidden, 1)
        act = gpu.act_empty(M, ffn, 1)
        linear(attn, wo, out_dev=h, op=_lib.EPI_RESID, resid_dev=h, ws=lws, M=M)
        rms_norm_rows(h, wo_ln, x, M, eps)
        linear(x, wgu, out_dev=act, op=_lib.EPI_SWIGLU, ws=lws, M=M)
        linear(act, wd, out_dev=h, op=_lib.EPI_RESID, resid_dev=h, ws=lws, M=M)
        return x, act

    wo_ln = ln
    h_ref = gpu.to_device(h0)
    x_ref, act_ref = four(h_ref)
    href = h_ref.to_numpy()
    x = gpu.act_empty(M, hidden, 1)
    act = gpu.act_empty(M, ffn, 1)
    for call in range(2):
        h = gpu.to_device(h0)
        mlp_block(attn, wo, h, ln, x, wgu, act, wd, M, eps, mws)
        gpu.device_synchronize()
        np.testing.assert_allclose(gpu.split_to_host(x, M), gpu.split_to_host(x_ref, M),
                                   rtol=1e-2, atol=1e-2, err_msg=f"x, call {call}")
        _close_mlp(h.to_numpy(), href, f"h, call {call}")
    h = gpu.to_device(h0)
    g = gpu.Graph()
    with g:
        mlp_block(attn, wo, h, ln, x, wgu, act, wd, M, eps, mws)
    for rep in range(3):
        gpu.copy_d2d(h, gpu.to_device(h0))
        g.launch()
        gpu.device_synchronize()
        _close_mlp(h.to_numpy(), href, f"h, replay {rep}")
    del g


def test_mlp_block_rejects_bad_shapes(gpu):
    from triton_llm.kernels.linear import Linear
    from triton_llm.kernels.mlp import MlpWorkspace, mlp_block
    with pytest.raises(ValueError):
        MlpWorkspace(65, 1024, 1024, 2048)        # more rows than a tile
    with pytest.raises(ValueError):
        MlpWorkspace(8, 1024, 1000, 2048)         # hidden not a multiple of 128
    ws = MlpWorkspace(8, 128, 128, 128)
    lin = Linear(np.zeros((128, 128), F32), "float32")
    a = gpu.act_empty(8, 128, 1)
    with pytest.raises(ValueError):               # fp32 weights
        mlp_block(a, lin, gpu.allocate((8, 128), np.float32), gpu.allocate((128,), np.float32),
                  a, lin, a, lin, 8, 1e-5, ws)


# ---------------------------------------------------------- folded RMSNorm --
@pytest.mark.parametrize("planes", [1, 2])
@pytest.mark.parametrize("M,N,K", [(64, 3072, 3072), (8, 576, 576), (33, 1000, 1536)])
def test_folded_norm_producer(gpu, monkeypatch, M, N, K, planes):
    """op RESID with a folded norm: h is what the plain RESID call on the
    same (tensor-core) kernel writes, bit for bit; fx = the operand format of
    h * w; the partial sums are the sums of squares of h over each 128-column
    weight tile."""
    from triton_llm import _lib
    monkeypatch.setenv("TLLM_SKINNY_MAX_M", "0")   # the plain call on tcgen05 too
    from triton_llm.kernels.linear import FoldedNorm, Linear, LinearWorkspace, linear
    rng = np.random.default_rng(M + N)
    lin = Linear((rng.standard_normal((N, K), dtype=F32) * 0.05).astype(F32), "bfloat16")
    x = gpu.to_device_split(rng.standard_normal((M, K), dtype=F32), planes=planes)
    h0 = rng.standard_normal((M, N), dtype=F32)
    wn = rng.standard_normal(N, dtype=F32)
    ws = LinearWorkspace([(M, N, K)])
    ha = gpu.to_device(h0)
    linear(x, lin, out_dev=ha, op=_lib.EPI_RESID, resid_dev=ha, ws=ws, M=M)
    hb = gpu.to_device(h0)
    fx = gpu.act_empty(M + 3, N, planes)
    ss = gpu.allocate((-(-N // 16), M + 5), np.float32)
    fold = FoldedNorm(gpu.to_device(wn), fx, ss, N, 1e-5, M, K)
    linear(x, lin, out_dev=hb, op=_lib.EPI_RESID, resid_dev=hb, ws=ws, M=M, fold_out=fold)
    h = hb.to_numpy()
    np.testing.assert_array_equal(h, ha.to_numpy())
    got_fx = gpu.split_to_host(fx, M)
    want_fx = (h * wn).astype(F32)
    if planes == 1:
        np.testing.assert_array_equal(got_fx, ops.bf16_round(want_fx))
    else:
        hi = ops.bf16_round(want_fx)
        np.testing.assert_array_equal(got_fx, hi + ops.bf16_round(want_fx - hi))
    from triton_llm.kernels.linear import fold_parts
    parts = fold_parts(M, N, K)
    width = 128      # folded calls run on the tensor-core kernel: one part per tile
    assert parts == -(-N // width)
    pad = np.zeros((M, parts * width), np.float64)
    pad[:, :N] = h.astype(np.float64) ** 2
    want_ss = pad.reshape(M, parts, width).sum(axis=2).T
    np.testing.assert_allclose(ss.to_numpy()[:parts, :M], want_ss, rtol=2e-6)


@pytest.mark.parametrize("planes", [1, 2])
@pytest.mark.parametrize("op", ["store", "swiglu", "qkv"])
@pytest.mark.parametrize("M", [8, 64])
def test_folded_norm_consumer(gpu, op, M, planes):
    """A projection reading h * w with the rows divided by their rms gives
    what RMSNorm followed by the plain projection gives (to the fp32 sums
    and the operand rounding of the two forms)."""
    from triton_llm import _lib
    from triton_llm.kernels.linear import (FoldedNorm, Linear, LinearWorkspace, linear,
                                           qkv_rows, swiglu_rows)
    from triton_llm.kernels.rms_norm import rms_norm_rows
    from triton_llm.kernels.rope import precompute_cos_sin
    rng = np.random.default_rng(7 * M + planes)
    n = 576
    h = (rng.standard_normal((M, n), dtype=F32) * 3).astype(F32)
    wn = (rng.standard_normal(n, dtype=F32) * 0.5 + 1).astype(F32)
    H, Hkv, D = 9, 3, 64
    if op == "swiglu":
        w = rng.standard_normal((2 * 1536, n), dtype=F32) * 0.05
        w = swiglu_rows(w[:1536], w[1536:])
    elif op == "qkv":
        w, _ = qkv_rows(rng.standard_normal((H * D, n), dtype=F32) * 0.05,
                        rng.standard_normal((Hkv * D, n), dtype=F32) * 0.05,
                        rng.standard_normal((Hkv * D, n), dtype=F32) * 0.05, D)
    else:
        w = rng.standard_normal((4096, n), dtype=F32) * 0.05
    lin = Linear(np.ascontiguousarray(w, F32), "bfloat16")
    code = {"store": _lib.EPI_STORE, "swiglu": _lib.EPI_SWIGLU, "qkv": _lib.EPI_QKV}[op]
    ws = LinearWorkspace([(M, lin.N, n)])
    hd, wd = gpu.to_device(h), gpu.to_device(wn)
    S = 16
    cos, sin = precompute_cos_sin(S, D, 1e5)
    cd, sd = gpu.to_device(cos), gpu.to_device(sin)
    seq = gpu.to_device(np.arange(M, dtype=np.int32))
    pos = gpu.to_device((np.arange(M) % S).astype(np.int32))

    def run(x, fold):
        if op == "qkv":
            q = gpu.allocate((M, H, D), np.float32)
            kc = gpu.zeros((M, Hkv, S, D), np.float32)
            vc = gpu.zeros((M, Hkv, S, D), np.float32)
            linear(x, lin, op=code, ws=ws, M=M, fold_in=fold, qkv=dict(
                cos=cd, sin=sd, row_seq=seq, row_pos=pos, q_out=q, k_cache=kc,
                v_cache=vc, n_head=H, n_kv_head=Hkv, head_dim=D))
            return np.concatenate([q.to_numpy().ravel(), kc.to_numpy().ravel(),
                                   vc.to_numpy().ravel()])
        out = gpu.allocate((M, lin.N // 2 if op == "swiglu" else lin.N), np.float32)
        linear(x, lin, out_dev=out, op=code, ws=ws, M=M, fold_in=fold)
        return out.to_numpy()

    # reference: RMSNorm kernel, then the plain projection
    xa = gpu.act_empty(M, n, planes)
    rms_norm_rows(hd, wd, xa, M, 1e-5)
    want = run(xa, None)
    # folded: the operand h * w and partial sums over 16-column parts (the
    # consumer adds whatever parts it is given)
    fx = gpu.to_device_split((h * wn).astype(F32), planes=planes)
    parts = n // 16
    ssh = (h.astype(F32) ** 2).reshape(M, parts, 16).sum(axis=2, dtype=F32).T.copy()
    ss = gpu.to_device(np.ascontiguousarray(ssh, F32))
    fold = FoldedNorm(wd, fx, ss, n, 1e-5, M, 576)
    fold.parts = parts
    got = run(fx, fold)
    scale = np.abs(want).max()
    tol = 2e-5 if planes == 2 else 2e-2
    np.testing.assert_allclose(got, want, atol=tol * scale)


def test_folded_norm_rejects_bad_use(gpu):
    from triton_llm import _lib
    from triton_llm.kernels.linear import FoldedNorm, Linear, LinearWorkspace, linear
    M, N = 4, 128
    lin = Linear(np.zeros((N, N), F32), "bfloat16")
    fx = gpu.act_empty(M, N, 2)
    fold = FoldedNorm(gpu.to_device(np.ones(N, F32)), fx, gpu.allocate((8, M), np.float32),
                      N, 1e-5, M, N)
    out = gpu.allocate((M, N), np.float32)
    with pytest.raises(ValueError):   # a producer must be op RESID
        linear(fx, lin, out_dev=out, op=_lib.EPI_STORE, M=M, fold_out=fold)
    with pytest.raises(ValueError):   # a consumer cannot be op RESID
        linear(fx, lin, out_dev=out, op=_lib.EPI_RESID, resid_dev=out, M=M, fold_in=fold)
