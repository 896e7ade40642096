"""Deterministic inputs shared by the golden generator and the tests.

Pure numpy; imports neither the reference nor the product package, so both
``gen_golden.py`` (which imports the reference) and the tests (which import
the product) can use it.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32


# ------------------------------------------------------------ model shapes ----
@dataclass(frozen=True)
class LlamaShape:
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    max_position_embeddings: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 100000.0

    def config_kwargs(self):
        return dict(vocab_size=self.vocab_size, hidden_size=self.hidden_size,
                    num_hidden_layers=self.num_hidden_layers,
                    num_attention_heads=self.num_attention_heads,
                    num_key_value_heads=self.num_key_value_heads,
                    intermediate_size=self.intermediate_size,
                    max_position_embeddings=self.max_position_embeddings,
                    rms_norm_eps=self.rms_norm_eps, rope_theta=self.rope_theta)


# the reference's tiny test model (tests/test_smollm2_model.py:46-54)
SMOL_TINY = LlamaShape(100, 64, 2, 4, 2, 128, 512)
# SmolLM2-135M, full depth
SMOL_135M = LlamaShape(49152, 576, 30, 9, 3, 1536, 8192, 1e-5, 100000.0)
# Llama-3.2-3B geometry with 2 of its 28 layers (parity slice of configs 4/5)
LLAMA3B_2L = LlamaShape(128256, 3072, 2, 24, 8, 8192, 8192, 1e-5, 500000.0)


def llama_weights_legacy(shape: LlamaShape, seed=42, scale=0.02):
    """Weights drawn like the reference's tiny-model test.

    np.random.seed(seed), then randn(...) * scale in this order: embedding,
    final norm, then per layer input norm, post-attention norm, q, k, v, o,
    gate, up, down (HF (out, in) layouts). Matches the draw order of
    tests/test_smollm2_model.py:14-40 so the reference's greedy tokens are
    reproducible.
    """
    n, v = shape.hidden_size, shape.vocab_size
    nh, nkv = shape.num_attention_heads, shape.num_key_value_heads
    dk = n // nh
    ffn = shape.intermediate_size
    rs = np.random.RandomState(seed)

    def r(*s):
        return rs.randn(*s).astype(F32) * F32(scale)

    w = {"model.embed_tokens.weight": r(v, n), "model.norm.weight": r(n)}
    for i in range(shape.num_hidden_layers):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = r(n)
        w[p + "post_attention_layernorm.weight"] = r(n)
        w[p + "self_attn.q_proj.weight"] = r(nh * dk, n)
        w[p + "self_attn.k_proj.weight"] = r(nkv * dk, n)
        w[p + "self_attn.v_proj.weight"] = r(nkv * dk, n)
        w[p + "self_attn.o_proj.weight"] = r(n, nh * dk)
        w[p + "mlp.gate_proj.weight"] = r(ffn, n)
        w[p + "mlp.up_proj.weight"] = r(ffn, n)
        w[p + "mlp.down_proj.weight"] = r(n, ffn)
    return w


def llama_weights(shape: LlamaShape, seed=0, std=0.02):
    """Random-init N(0, std) weights.

    ``np.random.default_rng(seed).standard_normal`` in HF state-dict order:
    embedding, then per layer q, k, v, o, gate, up, down, input norm,
    post-attention norm, then the final norm. Everything, norms included,
    is N(0, std) -- the literal reading of "random-init N(0,0.02)".
    """
    n, v = shape.hidden_size, shape.vocab_size
    nh, nkv = shape.num_attention_heads, shape.num_key_value_heads
    dk = n // nh
    ffn = shape.intermediate_size
    rng = np.random.default_rng(seed)

    def r(*s):
        return (rng.standard_normal(s, dtype=F32) * F32(std)).astype(F32)

    w = {"model.embed_tokens.weight": r(v, n)}
    for i in range(shape.num_hidden_layers):
        p = f"model.layers.{i}."
        w[p + "self_attn.q_proj.weight"] = r(nh * dk, n)
        w[p + "self_attn.k_proj.weight"] = r(nkv * dk, n)
        w[p + "self_attn.v_proj.weight"] = r(nkv * dk, n)
        w[p + "self_attn.o_proj.weight"] = r(n, nh * dk)
        w[p + "mlp.gate_proj.weight"] = r(ffn, n)
        w[p + "mlp.up_proj.weight"] = r(ffn, n)
        w[p + "mlp.down_proj.weight"] = r(n, ffn)
        w[p + "input_layernorm.weight"] = r(n)
        w[p + "post_attention_layernorm.weight"] = r(n)
    w["model.norm.weight"] = r(n)
    return w


# Llama-3.2-3B (BASELINE configs 4/5), full depth
LLAMA3B = LlamaShape(128256, 3072, 28, 24, 8, 8192, 8192, 1e-5, 500000.0)


def llama_keys(shape: LlamaShape):
    """HF state-dict keys of a Llama model, in ``llama_weights`` order, with
    their shapes."""
    n, v = shape.hidden_size, shape.vocab_size
    nh, nkv = shape.num_attention_heads, shape.num_key_value_heads
    dk, ffn = n // nh, shape.intermediate_size
    out = [("model.embed_tokens.weight", (v, n))]
    for i in range(shape.num_hidden_layers):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj.weight", (nh * dk, n)),
                (p + "self_attn.k_proj.weight", (nkv * dk, n)),
                (p + "self_attn.v_proj.weight", (nkv * dk, n)),
                (p + "self_attn.o_proj.weight", (n, nh * dk)),
                (p + "mlp.gate_proj.weight", (ffn, n)),
                (p + "mlp.up_proj.weight", (ffn, n)),
                (p + "mlp.down_proj.weight", (n, ffn)),
                (p + "input_layernorm.weight", (n,)),
                (p + "post_attention_layernorm.weight", (n,))]
    out.append(("model.norm.weight", (n,)))
    return out


class LazyLlamaWeights:
    """Random-init N(0, std) weights of a Llama model, generated when a key
    is read (so a 3B-parameter model never has to sit in host memory twice).

    Tensor ``i`` of ``llama_keys`` is ``default_rng([seed, i])
    .standard_normal`` times std; with ``bf16`` the matrices are rounded to
    bf16 (the weights the bf16 path stores exactly). Every read of a key
    gives the same values. Mapping-like: keys(), items(), [], in, len.
    """

    def __init__(self, shape: LlamaShape, seed=0, std=0.02, bf16=True):
        self.shape, self.seed, self.std, self.bf16 = shape, seed, std, bf16
        self._keys = llama_keys(shape)
        self._index = {k: (i, s) for i, (k, s) in enumerate(self._keys)}

    def __getitem__(self, key):
        i, shp = self._index[key]
        rng = np.random.default_rng([self.seed, i])
        a = (rng.standard_normal(shp, dtype=F32) * F32(self.std)).astype(F32)
        return bf16_round(a) if (self.bf16 and a.ndim == 2) else a

    def __contains__(self, key):
        return key in self._index

    def __len__(self):
        return len(self._keys)

    def __iter__(self):
        return iter(k for k, _ in self._keys)

    def keys(self):
        return [k for k, _ in self._keys]

    def items(self):
        return ((k, self[k]) for k, _ in self._keys)

    def get(self, key, default=None):
        return self[key] if key in self else default


DIGEST_COLS = 4096   # logit columns kept per step by logits_digest
DIGEST_TOPK = 32


def digest_columns(vocab, seed=12345):
    """The fixed, sorted logit columns a digest keeps (seeded, no repeats)."""
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(vocab, size=min(DIGEST_COLS, vocab), replace=False))


def logits_digest(logits):
    """Compact record of per-step logits (steps, V) of a long greedy run:
    the full rows of the first and last step, every step's values at
    ``digest_columns`` and its top-``DIGEST_TOPK`` (index, value) pairs in
    descending order, and each step's gap between its two largest logits
    (the margin its greedy token has)."""
    lg = np.asarray(logits, F32)
    cols = digest_columns(lg.shape[1])
    top = np.argsort(-lg, axis=1, kind="stable")[:, :DIGEST_TOPK]
    topv = np.take_along_axis(lg, top, axis=1)
    return {"first": lg[0].copy(), "last": lg[-1].copy(), "cols": cols,
            "at_cols": lg[:, cols].copy(), "top_idx": top.astype(np.int32),
            "top_val": topv, "gap": (topv[:, 0] - topv[:, 1]).astype(F32)}


def bf16_round(x):
    a = np.ascontiguousarray(x, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(F32).copy()


def round_linear_weights_bf16(weights: dict) -> dict:
    """bf16-round every matrix (Linear weights, embedding); keep 1-D norms."""
    return {k: (bf16_round(v) if np.ndim(v) == 2 else v) for k, v in weights.items()}


# ------------------------------------------------------------------ GPT-2 ----
@dataclass(frozen=True)
class GPT2Shape:
    vocab_size: int = 50257
    n_embd: int = 768
    n_layer: int = 12
    n_head: int = 12
    n_positions: int = 1024
    layer_norm_epsilon: float = 1e-5

    def config_kwargs(self):
        return dict(vocab_size=self.vocab_size, n_embd=self.n_embd,
                    n_layer=self.n_layer, n_head=self.n_head,
                    n_positions=self.n_positions,
                    layer_norm_epsilon=self.layer_norm_epsilon)


GPT2_TINY = GPT2Shape(100, 64, 2, 4, 1024)
GPT2_SMALL = GPT2Shape()


def gpt2_weights_legacy(shape: GPT2Shape, seed=42):
    """Draw order and scale of tests/test_gpt2_kv_cache.py:13-41 (randn, no
    scaling): wte, wpe, ln_f w/b, then per layer c_attn w/b, c_proj w/b,
    c_fc w/b, mlp c_proj w/b, ln_1 w/b, ln_2 w/b."""
    n, v = shape.n_embd, shape.vocab_size
    rs = np.random.RandomState(seed)

    def r(*s):
        return rs.randn(*s).astype(F32)

    w = {"wte.weight": r(v, n), "wpe.weight": r(shape.n_positions, n),
         "ln_f.weight": r(n), "ln_f.bias": r(n)}
    for i in range(shape.n_layer):
        p = f"h.{i}."
        w[p + "attn.c_attn.weight"] = r(n, 3 * n)
        w[p + "attn.c_attn.bias"] = r(3 * n)
        w[p + "attn.c_proj.weight"] = r(n, n)
        w[p + "attn.c_proj.bias"] = r(n)
        w[p + "mlp.c_fc.weight"] = r(n, 4 * n)
        w[p + "mlp.c_fc.bias"] = r(4 * n)
        w[p + "mlp.c_proj.weight"] = r(4 * n, n)
        w[p + "mlp.c_proj.bias"] = r(n)
        w[p + "ln_1.weight"] = r(n)
        w[p + "ln_1.bias"] = r(n)
        w[p + "ln_2.weight"] = r(n)
        w[p + "ln_2.bias"] = r(n)
    return w


def gpt2_weights(shape: GPT2Shape, seed=0, std=0.02):
    """every state-dict tensor N(0, std) from
    ``np.random.default_rng(seed)``, in HF GPT-2 order (wte, wpe, per layer
    ln_1 w/b, c_attn w/b, c_proj w/b, ln_2 w/b, c_fc w/b, mlp c_proj w/b,
    then ln_f w/b)."""
    n, v = shape.n_embd, shape.vocab_size
    rng = np.random.default_rng(seed)

    def r(*s):
        return (rng.standard_normal(s, dtype=F32) * F32(std)).astype(F32)

    w = {"wte.weight": r(v, n), "wpe.weight": r(shape.n_positions, n)}
    for i in range(shape.n_layer):
        p = f"h.{i}."
        w[p + "ln_1.weight"] = r(n)
        w[p + "ln_1.bias"] = r(n)
        w[p + "attn.c_attn.weight"] = r(n, 3 * n)
        w[p + "attn.c_attn.bias"] = r(3 * n)
        w[p + "attn.c_proj.weight"] = r(n, n)
        w[p + "attn.c_proj.bias"] = r(n)
        w[p + "ln_2.weight"] = r(n)
        w[p + "ln_2.bias"] = r(n)
        w[p + "mlp.c_fc.weight"] = r(n, 4 * n)
        w[p + "mlp.c_fc.bias"] = r(4 * n)
        w[p + "mlp.c_proj.weight"] = r(4 * n, n)
        w[p + "mlp.c_proj.bias"] = r(n)
    w["ln_f.weight"] = r(n)
    w["ln_f.bias"] = r(n)
    return w


# ------------------------------------------------- config 2 (isolated GQA) ----
def cfg2_inputs(seed=1, batch=64, n_head=9, n_kv=3, d=64, lo=128, hi=2048):
    """rng = default_rng(1); L = integers(128, 2049, 64);
    q (64, 9, 64); then per sequence K (3, L, 64), V (3, L, 64); all N(0,1),
    rounded to bf16 (returned as fp32 arrays holding bf16 values)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, batch).astype(np.int32)
    q = bf16_round(rng.standard_normal((batch, n_head, d), dtype=F32))
    ks, vs = [], []
    for L in lens:
        ks.append(bf16_round(rng.standard_normal((n_kv, int(L), d), dtype=F32)))
        vs.append(bf16_round(rng.standard_normal((n_kv, int(L), d), dtype=F32)))
    return lens, q, ks, vs


def pack_cache(seqs, max_seq):
    """List of (Hkv, L, d) arrays -> (B, Hkv, max_seq, d) zero-padded."""
    B = len(seqs)
    Hkv, _, d = seqs[0].shape
    out = np.zeros((B, Hkv, max_seq, d), F32)
    for b, s in enumerate(seqs):
        out[b, :, : s.shape[1]] = s
    return out


# ------------------------------------------------ temperature / top-k ----
@dataclass(frozen=True)
class SampleCase:
    """One call of the reference's ``_sample(logits, temperature, top_k)``
    after ``np.random.seed(rng)``: logits = N(0,1) * scale (default_rng(seed),
    float32) of length V."""
    seed: int
    V: int
    scale: float
    temperature: float
    top_k: int
    rng: int


def _sample_cases():
    vocabs = (100, 49152, 50257, 128256)
    temps = (0.3, 0.7, 1.0, 1.5)
    ks = (0, 1, 5, 50, 1000, -1, -2)   # -1: top_k = V, -2: top_k = V + 7
    scales = (1.0, 3.0, 8.0)
    out = []
    for i in range(48):
        V = vocabs[i % 4]
        k = ks[(i // 4) % 7]
        k = V if k == -1 else V + 7 if k == -2 else min(k, V)
        out.append(SampleCase(seed=100 + i, V=V, scale=scales[i % 3],
                              temperature=temps[(i // 2) % 4], top_k=k,
                              rng=1000 + i))
    return tuple(out)


SAMPLE_CASES = _sample_cases()


def sample_logits(case: SampleCase) -> np.ndarray:
    rng = np.random.default_rng(case.seed)
    return (rng.standard_normal(case.V, dtype=F32) * F32(case.scale)).astype(F32)


def sample_uniform(rng_seed: int, n: int = 1) -> np.ndarray:
    """The uniforms np.random.choice draws after np.random.seed(rng_seed):
    one random_sample() per call, from the legacy global generator."""
    return np.random.RandomState(rng_seed).random_sample(n)
