"""Pin the CPU oracle against the reference's own outputs (CPU only).

The fixtures in tests/golden/ were produced by running the reference
triton-llm (its Triton kernels under TRITON_INTERPRET=1) by
tests/golden/gen_golden.py. These tests check that the numpy restatement in
``oracle/`` reproduces them, so it can serve as the checker for the CUDA
path. Tolerances are the reference tests' own (atol 1e-4 for attention,
tests/test_attention_gqa.py:144; 1e-4 for RoPE/RMSNorm/SwiGLU).
"""

from __future__ import annotations

import numpy as np
import pytest

import inputs
from oracle import models, ops

F32 = np.float32


def _cases(g, prefix):
    keys = sorted({k.split("/")[1] for k in g if k.startswith(prefix + "/")})
    return keys


def test_gqa_matches_reference(golden):
    g = golden("kernels")
    names = _cases(g, "gqa")
    assert len(names) >= 10
    for n in names:
        nh, nkv, causal = (int(x) for x in g[f"gqa/{n}/meta"])
        out = ops.gqa_attention(g[f"gqa/{n}/q"], g[f"gqa/{n}/k"], g[f"gqa/{n}/v"],
                                nh, nkv, causal=bool(causal))
        np.testing.assert_allclose(out, g[f"gqa/{n}/out"], atol=1e-5, rtol=1e-5,
                                   err_msg=n)


def test_gqa_decode_batched_equals_flat(golden):
    g = golden("kernels")
    # pack the config-2 geometry cases into one ragged batch
    names = [n for n in _cases(g, "gqa") if n.startswith("decode_9_3_64_L")]
    seqs_k = [g[f"gqa/{n}/k"].reshape(3, -1, 64) for n in names]
    seqs_v = [g[f"gqa/{n}/v"].reshape(3, -1, 64) for n in names]
    lens = np.array([s.shape[1] for s in seqs_k])
    q = np.stack([g[f"gqa/{n}/q"] for n in names])
    out = ops.gqa_decode(q, inputs.pack_cache(seqs_k, lens.max()),
                         inputs.pack_cache(seqs_v, lens.max()), lens)
    for i, n in enumerate(names):
        np.testing.assert_allclose(out[i], g[f"gqa/{n}/out"], atol=1e-5,
                                   rtol=1e-5)


def test_gqa_empty():
    # tests/test_attention_gqa.py:272-308
    q = np.zeros((0, 64), F32)
    k = np.random.randn(16, 64).astype(F32)
    assert ops.gqa_attention(q, k, k, 4, 2, causal=False).shape == (0, 64)
    out = ops.gqa_attention(np.ones((16, 64), F32), np.zeros((0, 64), F32),
                            np.zeros((0, 64), F32), 4, 2, causal=False)
    assert out.shape == (16, 64) and np.all(out == 0)


def test_rope_tables_bit_exact(golden):
    g = golden("kernels")
    for theta in (10000, 100000, 500000):
        for d in (64, 128):
            c, s = ops.precompute_cos_sin(64, d, float(theta))
            np.testing.assert_array_equal(c, g[f"rope/table/{theta}/{d}/cos"])
            np.testing.assert_array_equal(s, g[f"rope/table/{theta}/{d}/sin"])


def test_rope_apply(golden):
    g = golden("kernels")
    c, s = ops.precompute_cos_sin(256, 64, 100000.0)
    for key in [k for k in g if k.startswith("rope/apply/") and k.endswith("/x")]:
        name = key.split("/")[2]
        if name.endswith("_d128"):
            cc, ss = ops.precompute_cos_sin(8192, 128, 500000.0)
            rows, seq, off = 32, 1, 8000
        else:
            cc, ss = c, s
            rows, seq, off = (int(v) for v in name.split("_"))
        out = ops.apply_rope(g[key], cc, ss, seq, off)
        np.testing.assert_allclose(out, g[key[:-2] + "/out"], atol=1e-6,
                                   rtol=1e-6, err_msg=name)


def test_rope_identity_at_pos0():
    # tests/test_rope.py:75-103: position 0 is the identity
    c, s = ops.precompute_cos_sin(16, 64, 100000.0)
    x = np.random.randn(9, 64).astype(F32)
    np.testing.assert_array_equal(ops.apply_rope(x, c, s, 1, 0), x)


def test_rms_norm(golden):
    g = golden("kernels")
    for (m, n) in ((4, 576), (3, 777), (2, 1), (1, 3072)):
        out = ops.rms_norm(g[f"rms/{m}_{n}/x"], g[f"rms/{m}_{n}/w"], 1e-5)
        np.testing.assert_allclose(out, g[f"rms/{m}_{n}/out"], atol=1e-5,
                                   rtol=1e-5)
    # tests/test_rms_norm.py:74-82: x = 3, w = 2 -> 2
    known = ops.rms_norm(np.array([[3.0]], F32), np.array([2.0], F32))
    np.testing.assert_allclose(known, g["rms/known/out"], atol=1e-6)
    np.testing.assert_allclose(known, [[2.0]], atol=1e-5)


def test_elementwise(golden):
    g = golden("kernels")
    with np.errstate(over="ignore", invalid="ignore"):
        np.testing.assert_allclose(ops.swiglu(g["swiglu/x"], g["swiglu/y"]),
                                   g["swiglu/out"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(ops.gelu(g["gelu/x"]), g["gelu/out"],
                                   rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(ops.add(g["add/x"], g["add/y"]), g["add/out"])
    # tests/test_swiglu.py:86-95: silu(3) * 2 = 6 / (1 + e^-3) = 5.71544
    assert abs(float(ops.swiglu(np.float32([3.0]), np.float32([2.0]))[0]) - 5.715445) < 1e-5


def test_layer_norm_and_embedding(golden):
    g = golden("kernels")
    for (m, n) in ((3, 768), (2, 100)):
        out = ops.layer_norm(g[f"ln/{m}_{n}/x"], g[f"ln/{m}_{n}/g"],
                             g[f"ln/{m}_{n}/b"], 1e-5)
        np.testing.assert_allclose(out, g[f"ln/{m}_{n}/out"], atol=1e-5,
                                   rtol=1e-5)
    emb = ops.embedding(g["emb/ids"], g["emb/wte"], g["emb/wpe"], 9)
    np.testing.assert_array_equal(emb, g["emb/out"])


def test_gemm(golden):
    g = golden("kernels")
    for (m, k, n) in ((1, 576, 192), (3, 64, 100), (5, 130, 70)):
        out = ops.gemm(g[f"gemm/{m}_{k}_{n}/a"], g[f"gemm/{m}_{k}_{n}/b"])
        np.testing.assert_allclose(out, g[f"gemm/{m}_{k}_{n}/out"], atol=1e-5,
                                   rtol=1e-5)


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8,
                  3.0e38, 1e-40], F32)
    r = ops.bf16_round(x)
    assert r[0] == 1.0
    assert r[1] == 1.0                      # tie -> even (down)
    assert r[2] == 1.0 + 4 * 2 ** -8        # tie -> even (up)
    assert r[3] == -1.0
    assert np.all((r.view(np.uint32) & 0xFFFF) == 0)


# ------------------------------------------------------------------ models ----
class _Cfg:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def test_smol_tiny_matches_reference(golden):
    g = golden("smol_tiny")
    shape = inputs.SMOL_TINY
    w = inputs.llama_weights_legacy(shape, seed=42)
    orc = models.SmolLM2Oracle(_Cfg(**shape.config_kwargs()), w)
    toks, logits = orc.generate([5, 12, 7], 5)
    np.testing.assert_array_equal(toks[0], g["tokens"])
    assert g["tokens"].tolist() == [5, 12, 7, 72, 86, 92, 86, 92]
    np.testing.assert_allclose(logits, g["logits"], atol=1e-6, rtol=1e-5)


def test_gpt2_tiny_matches_reference(golden):
    g = golden("gpt2_tiny")
    shape = inputs.GPT2_TINY
    w = inputs.gpt2_weights_legacy(shape, seed=42)
    orc = models.GPT2Oracle(_Cfg(**shape.config_kwargs()), w)
    toks, logits = orc.generate([5, 12, 7, 0, 3], 10)
    np.testing.assert_array_equal(toks[0], g["tokens"])
    # randn weights give logits of order 1e2-1e3: relative tolerance
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("name,shape,n_new,vocab", [
    ("smol135m_slice", inputs.SMOL_135M, 3, 49152),
    ("llama3b_2l_slice", inputs.LLAMA3B_2L, 2, 128256),
])
def test_full_geometry_slices(golden, name, shape, n_new, vocab):
    """Full-width SmolLM2-135M / Llama-3.2-3B layers: the oracle with bf16
    weights and fp32 K/V reproduces the reference run on the same weights."""
    g = golden(name)
    w = inputs.round_linear_weights_bf16(inputs.llama_weights(shape, 0))
    prompt = g["tokens"][: len(g["tokens"]) - n_new].tolist()
    orc = models.SmolLM2Oracle(_Cfg(**shape.config_kwargs()), w,
                               weight_dtype="float32", kv_dtype="float32")
    toks, logits = orc.generate(prompt, n_new)
    np.testing.assert_array_equal(toks[0], g["tokens"])
    np.testing.assert_allclose(logits, g["logits"], atol=1e-4)


def test_gpt2_small_slice(golden):
    g = golden("gpt2_small_slice")
    shape = inputs.GPT2_SMALL
    w = inputs.gpt2_weights(shape, 0)
    orc = models.GPT2Oracle(_Cfg(**shape.config_kwargs()), w)
    prompt = g["tokens"][:-2].tolist()
    toks, logits = orc.generate(prompt, 2)
    np.testing.assert_array_equal(toks[0], g["tokens"])
    np.testing.assert_allclose(logits, g["logits"], atol=1e-4)


def test_gpt2_cfg1_32_steps(golden):
    """BASELINE config 1 (32-token prompt, 32 greedy steps): the oracle
    reproduces the reference's own tokens and, at the digest's columns and
    top-32 indices, its logits."""
    g = golden("gpt2_cfg1")
    shape = inputs.GPT2_SMALL
    orc = models.GPT2Oracle(_Cfg(**shape.config_kwargs()), inputs.gpt2_weights(shape, 0))
    toks, logits = orc.generate(g["tokens"][:32].tolist(), 32)
    np.testing.assert_array_equal(toks[0], g["tokens"])
    np.testing.assert_allclose(logits[0], g["first"], atol=1e-4)
    np.testing.assert_allclose(logits[-1], g["last"], atol=1e-4)
    np.testing.assert_allclose(logits[:, g["cols"]], g["at_cols"], atol=1e-4)
    np.testing.assert_allclose(np.take_along_axis(logits, g["top_idx"], axis=1),
                               g["top_val"], atol=1e-4)


# ------------------------------------------------ temperature / top-k ----
def test_sample_matches_reference_cases(golden):
    """The oracle's sampler picks the reference _sample's token on every
    case (vocabularies 100 to 128256; T 0.3 to 1.5; top_k 0, 1, 5, 50, 1000,
    V and V + 7), with the uniform np.random.choice draws after the case's
    np.random.seed."""
    g = golden("sample")
    for c, want in zip(inputs.SAMPLE_CASES, g["case_tokens"]):
        u = inputs.sample_uniform(c.rng)[0]
        got = ops.sample(inputs.sample_logits(c), c.temperature, c.top_k, u)
        assert got == int(want), (c, got, int(want))


def test_sample_replays_reference_sampled_run(golden):
    """The reference's tiny SmolLM2 generate at T=0.8, top_k=20 after
    np.random.seed(7): the oracle sampler on the reference's own per-step
    logits with the generator's successive uniforms gives its tokens."""
    g = golden("sample")
    T, k, seed = g["tiny_meta"]
    steps = g["tiny_logits"]
    us = inputs.sample_uniform(int(seed), len(steps))
    got = [ops.sample(lg, float(T), int(k), u) for lg, u in zip(steps, us)]
    np.testing.assert_array_equal(got, g["tiny_tokens"][3:])


def test_sample_properties():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(1000) * 3).astype(F32)
    # top_k = 1 is the argmax whatever u is
    for u in (0.0, 0.3, 0.999999):
        assert ops.sample(x, 0.7, 1, u) == int(np.argmax(x))
    # u = 0 picks the first index with positive weight; u -> 1 the last one
    assert ops.sample(x, 1.0, 0, 0.0) == 0
    assert ops.sample(x, 1.0, 0, np.nextafter(1.0, 0.0)) == 999
    # equal logits at the top_k threshold: the lowest indices are kept
    y = np.zeros(10, F32)
    y[[2, 5, 7]] = 1.0
    picks = {ops.sample(y, 1.0, 2, u) for u in np.linspace(0, 0.999, 50)}
    assert picks == {2, 5}
    # the cdf is monotone, ends at 1 and its steps are the kept weights
    cdf = ops.sample_cdf(x, 0.7, 50)
    assert np.all(np.diff(cdf) >= 0) and cdf[-1] == 1.0
    assert np.count_nonzero(np.diff(np.concatenate([[0.0], cdf]))) == 50
