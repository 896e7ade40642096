"""Generate golden vectors by running the reference triton-llm on the CPU.

    python tests/golden/gen_golden.py [--only NAME ...] [--slow]

The reference (a read-only checkout whose path is given in
$TLLM_REFERENCE) is imported with its GPU allocator replaced by a host-memory
stand-in and its Triton kernels run under TRITON_INTERPRET=1 (see
ref_shim.py). Inputs come from inputs.py. Every output is the reference's
own result; nothing here calls the oracle or the B200 product.

Fixtures written next to this script (small .npz files, committed):
  kernels.npz        per-kernel cases (GQA decode/prefill, RoPE, RMSNorm,
                     SwiGLU, GELU, LayerNorm, embedding, add, gemm)
  smol_tiny.npz      tiny SmolLM2 greedy run (tests/test_smollm2_model.py
                     model): prompt [5,12,7] + 5 tokens, per-step logits
  gpt2_tiny.npz      tiny GPT-2 greedy run (tests/test_gpt2_kv_cache.py
                     model): prompt [5,12,7,0,3] + 10 tokens
  smol135m_slice.npz SmolLM2-135M geometry, N(0,0.02) weights seed 0 rounded
                     to bf16, 8-token prompt + 3 greedy steps
  llama3b_2l_slice.npz Llama-3.2-3B geometry (2 layers), N(0,0.02) seed 0
                     rounded to bf16, 4-token prompt + 2 greedy steps
  gpt2_small_slice.npz (--slow) GPT-2 small N(0,0.02) seed 0, 8-token
                     prompt + 2 greedy steps
  sample.npz         the reference's _sample (temperature / top-k) on
                     inputs.SAMPLE_CASES after np.random.seed(case.rng),
                     and a tiny SmolLM2 run sampled at T=0.8, top_k=20
                     (np.random.seed(7)): tokens and per-step logits
  gpt2_cfg1.npz      (--slow) BASELINE config 1: GPT-2 small N(0,0.02) seed
                     0, 32-token prompt + 32 greedy steps; tokens and a
                     digest of the per-step logits (inputs.logits_digest)
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import inputs  # noqa: E402
import ref_shim  # noqa: E402

F32 = np.float32


def _log(msg):
    print(f"[gen_golden {time.strftime('%H:%M:%S')}] {msg}", flush=True)


def kernels_cases(g):
    from triton_llm.kernels.attention_gqa import attention_gqa
    from triton_llm.kernels.rope import precompute_cos_sin, apply_rope
    from triton_llm.kernels.rms_norm import rms_norm
    from triton_llm.kernels.swiglu import swiglu
    from triton_llm.kernels.gelu import gelu
    from triton_llm.kernels.layernorm import layer_norm
    from triton_llm.kernels.embedding import embedding
    from triton_llm.kernels.add import add
    from triton_llm.kernels.gemm import gemm

    out = {}

    def gqa(name, q, k, v, nh, nkv, causal):
        o = attention_gqa(g.to_device(q), g.to_device(k), g.to_device(v), nh,
                          nkv, causal=causal)
        out[f"gqa/{name}/q"] = q
        out[f"gqa/{name}/k"] = k
        out[f"gqa/{name}/v"] = v
        out[f"gqa/{name}/meta"] = np.array([nh, nkv, int(causal)], np.int32)
        out[f"gqa/{name}/out"] = o.to_numpy()

    # decode case of tests/test_attention_gqa.py:242-269 (9/3/64, L=16)
    rs = np.random.RandomState(42)
    q = rs.randn(9, 64).astype(F32)
    k = rs.randn(3 * 16, 64).astype(F32)
    v = rs.randn(3 * 16, 64).astype(F32)
    gqa("decode_9_3_64_L16", q, k, v, 9, 3, False)
    # decode at the config-2 head geometry, bf16-valued inputs, ragged edges
    rng = np.random.default_rng(7)
    for L in (1, 63, 64, 65, 200, 1031):
        q = inputs.bf16_round(rng.standard_normal((9, 64), dtype=F32))
        k = inputs.bf16_round(rng.standard_normal((3 * L, 64), dtype=F32))
        v = inputs.bf16_round(rng.standard_normal((3 * L, 64), dtype=F32))
        gqa(f"decode_9_3_64_L{L}", q, k, v, 9, 3, False)
    # Llama-3.2-3B head geometry (24/8/128) and MHA (GPT-2 style, 12/12/64)
    for (nh, nkv, d, L) in ((24, 8, 128, 300), (12, 12, 64, 77), (6, 2, 128, 129)):
        q = inputs.bf16_round(rng.standard_normal((nh, d), dtype=F32))
        k = inputs.bf16_round(rng.standard_normal((nkv * L, d), dtype=F32))
        v = inputs.bf16_round(rng.standard_normal((nkv * L, d), dtype=F32))
        gqa(f"decode_{nh}_{nkv}_{d}_L{L}", q, k, v, nh, nkv, False)
    # causal prefill cases of tests/test_attention_gqa.py:126-131 and :222-228
    rs = np.random.RandomState(42)
    for (nh, nkv, d, seq) in ((9, 3, 64, 8), (15, 5, 64, 8), (32, 8, 64, 16),
                              (6, 2, 128, 8), (9, 3, 64, 100)):
        q = rs.randn(nh * seq, d).astype(F32)
        k = rs.randn(nkv * seq, d).astype(F32)
        v = rs.randn(nkv * seq, d).astype(F32)
        gqa(f"prefill_{nh}_{nkv}_{d}_S{seq}", q, k, v, nh, nkv, True)
    q = rs.randn(6 * 2, 64).astype(F32)
    k = rs.randn(2 * 8, 64).astype(F32)
    v = rs.randn(2 * 8, 64).astype(F32)
    gqa("causal_sq2_sk8", q, k, v, 6, 2, True)

    # RoPE tables and rotations (rope.py:73-123, :153-222)
    for theta in (10000.0, 100000.0, 500000.0):
        for d in (64, 128):
            c, s = precompute_cos_sin(64, d, theta=theta)
            out[f"rope/table/{int(theta)}/{d}/cos"] = c
            out[f"rope/table/{int(theta)}/{d}/sin"] = s
    c, s = precompute_cos_sin(256, 64, theta=100000.0)
    for (rows, seq, off) in ((576, 8, 0), (9, 1, 37), (3, 1, 200), (144, 16, 5)):
        x = rs.randn(rows, 64).astype(F32)
        xd = g.to_device(x)
        apply_rope(xd, g.to_device(c), g.to_device(s), seq_len=seq,
                   position_offset=off)
        out[f"rope/apply/{rows}_{seq}_{off}/x"] = x
        out[f"rope/apply/{rows}_{seq}_{off}/out"] = xd.to_numpy()
    c, s = precompute_cos_sin(8192, 128, theta=500000.0)
    x = rs.randn(32, 128).astype(F32)
    xd = g.to_device(x)
    apply_rope(xd, g.to_device(c), g.to_device(s), seq_len=1, position_offset=8000)
    out["rope/apply/32_1_8000_d128/x"] = x
    out["rope/apply/32_1_8000_d128/out"] = xd.to_numpy()

    # RMSNorm widths of tests/test_rms_norm.py:19-27 plus the known answer
    for (m, n) in ((4, 576), (3, 777), (2, 1), (1, 3072)):
        x = rs.randn(m, n).astype(F32)
        w = rs.randn(n).astype(F32)
        o = g.allocate((m, n), np.float32)
        rms_norm(g.to_device(x), g.to_device(w), o, 1e-5)
        out[f"rms/{m}_{n}/x"], out[f"rms/{m}_{n}/w"] = x, w
        out[f"rms/{m}_{n}/out"] = o.to_numpy()
    o = g.allocate((1, 1), np.float32)
    rms_norm(g.to_device(np.array([[3.0]], F32)), g.to_device(np.array([2.0], F32)),
             o, 1e-5)
    out["rms/known/out"] = o.to_numpy()

    # SwiGLU / GELU / add (elementwise)
    x = np.concatenate([rs.randn(1000).astype(F32) * 4,
                        np.array([0.0, -0.0, 30.0, -30.0, 88.0, -88.0, 1e10, -1e10], F32)])
    y = rs.randn(x.size).astype(F32)
    out["swiglu/x"], out["swiglu/y"] = x, y
    out["swiglu/out"] = swiglu(g.to_device(x), g.to_device(y)).to_numpy()
    out["gelu/x"] = x
    out["gelu/out"] = gelu(x)
    out["add/x"], out["add/y"] = x, y
    out["add/out"] = add(g.to_device(x), g.to_device(y)).to_numpy()

    # LayerNorm (GPT-2)
    for (m, n) in ((3, 768), (2, 100)):
        x = (rs.randn(m, n) * 3 + 1).astype(F32)
        gm = rs.randn(n).astype(F32)
        bt = rs.randn(n).astype(F32)
        out[f"ln/{m}_{n}/x"], out[f"ln/{m}_{n}/g"], out[f"ln/{m}_{n}/b"] = x, gm, bt
        out[f"ln/{m}_{n}/out"] = layer_norm(x, gm, bt, 1e-5)

    # embedding with a position offset
    wte = rs.randn(100, 64).astype(F32)
    wpe = rs.randn(128, 64).astype(F32)
    ids = np.array([[5, 12, 7, 99, 0]], np.int32)
    out["emb/wte"], out["emb/wpe"], out["emb/ids"] = wte, wpe, ids
    out["emb/out"] = embedding(ids, wte, wpe, position_offset=9)

    # gemm: decode shapes (M=1) and a small prefill shape
    for (m, k, n) in ((1, 576, 192), (3, 64, 100), (5, 130, 70)):
        a = rs.randn(m, k).astype(F32)
        b = (rs.randn(k, n) * 0.05).astype(F32)
        out[f"gemm/{m}_{k}_{n}/a"], out[f"gemm/{m}_{k}_{n}/b"] = a, b
        out[f"gemm/{m}_{k}_{n}/out"] = gemm(g.to_device(a), g.to_device(b)).to_numpy()
    return out


def smol_run(shape, weights, prompt, n_new):
    from smollm2_triton.config import SmolLM2Config
    from smollm2_triton.model import SmolLM2ForCausalLM
    cfg = SmolLM2Config(**shape.config_kwargs())
    model = SmolLM2ForCausalLM(cfg, weights)
    model._init_cache_gpu(max_seq=len(prompt) + n_new)
    ids = np.array([prompt], np.int32)
    logits = model._forward_cached(ids)
    toks = list(prompt)
    steps = []
    for step in range(n_new):
        last = logits[0, -1]
        steps.append(last.copy())
        t = int(np.argmax(last))
        toks.append(t)
        if step < n_new - 1:
            logits = model._forward_cached(np.array([[t]], np.int32))
    return np.array(toks, np.int32), np.stack(steps)


def smol_sampled_run(shape, weights, prompt, n_new, temperature, top_k, seed):
    """The reference's generate loop (model.py:455-469) with sampling, after
    np.random.seed(seed); keeps the per-step logits."""
    from smollm2_triton.config import SmolLM2Config
    from smollm2_triton.model import SmolLM2ForCausalLM
    cfg = SmolLM2Config(**shape.config_kwargs())
    model = SmolLM2ForCausalLM(cfg, weights)
    model._init_cache_gpu(max_seq=len(prompt) + n_new)
    np.random.seed(seed)
    logits = model._forward_cached(np.array([prompt], np.int32))
    toks = list(prompt)
    steps = []
    for step in range(n_new):
        last = logits[0, -1]
        steps.append(last.copy())
        t = model._sample(last, temperature, top_k)
        toks.append(t)
        if step < n_new - 1:
            logits = model._forward_cached(np.array([[t]], np.int32))
    return np.array(toks, np.int32), np.stack(steps)


def sample_cases():
    """The reference's _sample on each of inputs.SAMPLE_CASES."""
    from smollm2_triton.model import SmolLM2ForCausalLM
    toks = []
    for c in inputs.SAMPLE_CASES:
        np.random.seed(c.rng)
        toks.append(SmolLM2ForCausalLM._sample(None, inputs.sample_logits(c),
                                               c.temperature, c.top_k))
    return np.array(toks, np.int64)


def gpt2_run(shape, weights, prompt, n_new):
    from gpt2_triton.config import GPT2Config
    from gpt2_triton.model import GPT2Model
    cfg = GPT2Config(**shape.config_kwargs())
    model = GPT2Model(cfg, weights)
    model._init_cache()
    logits = model.forward(np.array([prompt], np.int32), use_cache=True)
    toks = list(prompt)
    steps = []
    for step in range(n_new):
        last = logits[0, -1]
        steps.append(last.copy())
        t = int(np.argmax(last))
        toks.append(t)
        if step < n_new - 1:
            logits = model.forward(np.array([[t]], np.int32), use_cache=True)
    return np.array(toks, np.int32), np.stack(steps)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*", default=None)
    ap.add_argument("--slow", action="store_true")
    a = ap.parse_args()
    g = ref_shim.install()
    want = lambda n: a.only is None or n in a.only  # noqa: E731

    if want("kernels"):
        _log("kernels")
        np.savez_compressed(HERE / "kernels.npz", **kernels_cases(g))
    if want("smol_tiny"):
        _log("smol_tiny")
        w = inputs.llama_weights_legacy(inputs.SMOL_TINY, seed=42)
        toks, logits = smol_run(inputs.SMOL_TINY, w, [5, 12, 7], 5)
        _log(f"  tokens {toks.tolist()}")
        np.savez_compressed(HERE / "smol_tiny.npz", tokens=toks, logits=logits)
    if want("sample"):
        _log("sample")
        case_tokens = sample_cases()
        w = inputs.llama_weights_legacy(inputs.SMOL_TINY, seed=42)
        toks, logits = smol_sampled_run(inputs.SMOL_TINY, w, [5, 12, 7], 16,
                                        0.8, 20, 7)
        _log(f"  cases {case_tokens.tolist()}")
        _log(f"  tiny sampled tokens {toks.tolist()}")
        np.savez_compressed(HERE / "sample.npz", case_tokens=case_tokens,
                            tiny_tokens=toks, tiny_logits=logits,
                            tiny_meta=np.array([0.8, 20, 7], np.float64))
    if want("gpt2_tiny"):
        _log("gpt2_tiny")
        w = inputs.gpt2_weights_legacy(inputs.GPT2_TINY, seed=42)
        toks, logits = gpt2_run(inputs.GPT2_TINY, w, [5, 12, 7, 0, 3], 10)
        _log(f"  tokens {toks.tolist()}")
        np.savez_compressed(HERE / "gpt2_tiny.npz", tokens=toks, logits=logits)
    if want("smol135m_slice"):
        _log("smol135m_slice")
        w = inputs.round_linear_weights_bf16(inputs.llama_weights(inputs.SMOL_135M, 0))
        prompt = np.random.default_rng(0).integers(0, 49152, 8).tolist()
        toks, logits = smol_run(inputs.SMOL_135M, w, prompt, 3)
        _log(f"  tokens {toks.tolist()}")
        np.savez_compressed(HERE / "smol135m_slice.npz", tokens=toks, logits=logits)
    if want("llama3b_2l_slice"):
        _log("llama3b_2l_slice")
        w = inputs.round_linear_weights_bf16(inputs.llama_weights(inputs.LLAMA3B_2L, 0))
        prompt = np.random.default_rng(0).integers(0, 128256, 4).tolist()
        toks, logits = smol_run(inputs.LLAMA3B_2L, w, prompt, 2)
        _log(f"  tokens {toks.tolist()}")
        np.savez_compressed(HERE / "llama3b_2l_slice.npz", tokens=toks,
                            logits=logits)
    if a.slow and want("gpt2_small_slice"):
        _log("gpt2_small_slice")
        w = inputs.gpt2_weights(inputs.GPT2_SMALL, 0)
        prompt = np.random.default_rng(0).integers(0, 50257, 8).tolist()
        toks, logits = gpt2_run(inputs.GPT2_SMALL, w, prompt, 2)
        _log(f"  tokens {toks.tolist()}")
        np.savez_compressed(HERE / "gpt2_small_slice.npz", tokens=toks,
                            logits=logits)
    if a.slow and want("gpt2_cfg1"):
        # BASELINE config 1 as stated: GPT-2 small, N(0,0.02) seed-0 weights,
        # 32-token prompt (default_rng(0)), 32 greedy steps. About an hour of
        # CPU under the interpreter.
        _log("gpt2_cfg1")
        w = inputs.gpt2_weights(inputs.GPT2_SMALL, 0)
        prompt = np.random.default_rng(0).integers(0, 50257, 32).tolist()
        toks, logits = gpt2_run(inputs.GPT2_SMALL, w, prompt, 32)
        _log(f"  tokens {toks.tolist()}")
        np.savez_compressed(HERE / "gpt2_cfg1.npz", tokens=toks,
                            **inputs.logits_digest(logits))
    _log("done")


if __name__ == "__main__":
    main()
