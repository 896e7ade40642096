"""Numpy restatement of the reference kernels (test infrastructure only).

Each function follows one reference kernel line by line, in fp32, with the
same operation order where it changes rounding (division vs multiplication,
where the scale is applied, blockwise online softmax). Paths are inside
ziliangpeng/triton-llm.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


# ----------------------------------------------------------------- bf16 ----
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 value (ties to even), returned as fp32.

    This is the storage rounding the B200 path applies to weights and to K/V
    at cache append; the reference itself is fp32 only.
    """
    a = np.ascontiguousarray(x, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(F32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) of ``bf16_round(x)``."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# ------------------------------------------------------------ attention ----
def gqa_attention(q_flat, k_flat, v_flat, n_head, n_kv_head, causal=True,
                  sm_scale=None, block=64):
    """GQA attention, flat head-major layout.

    Follows triton_llm/kernels/attention_gqa.py:
      * kv head of q head h: h // (n_head // n_kv_head)      (:76)
      * q scaled once by sm_scale before the dot products   (:83)
      * keys in blocks of 64, online softmax in fp32         (:105-140)
      * causal: key j visible iff j <= seq_k - seq_q + i     (:97, :109-112)
      * one division by the running sum at the end          (:143)
    Shapes: q (n_head*seq_q, d), k/v (n_kv_head*seq_k, d) -> (n_head*seq_q, d).
    """
    q_flat = np.asarray(q_flat, F32)
    k_flat = np.asarray(k_flat, F32)
    v_flat = np.asarray(v_flat, F32)
    d = q_flat.shape[1]
    seq_q = q_flat.shape[0] // n_head
    seq_k = k_flat.shape[0] // n_kv_head
    if seq_q == 0:
        return np.zeros((0, d), F32)
    if seq_k == 0:
        return np.zeros((n_head * seq_q, d), F32)
    if sm_scale is None:
        sm_scale = 1.0 / (d ** 0.5)
    group = n_head // n_kv_head
    q = q_flat.reshape(n_head, seq_q, d) * F32(sm_scale)
    k = k_flat.reshape(n_kv_head, seq_k, d)
    v = v_flat.reshape(n_kv_head, seq_k, d)
    kv_of = np.arange(n_head) // group
    acc = np.zeros((n_head, seq_q, d), F32)
    row_max = np.full((n_head, seq_q), -np.inf, F32)
    row_sum = np.zeros((n_head, seq_q), F32)
    abs_q = seq_k - seq_q + np.arange(seq_q)
    with np.errstate(invalid="ignore", over="ignore"):
        for start in range(0, seq_k, block):
            stop = min(start + block, seq_k)
            kb = k[kv_of, start:stop]          # (H, n, d)
            vb = v[kv_of, start:stop]
            s = np.einsum("hqd,hnd->hqn", q, kb, dtype=F32)
            offs = np.arange(start, stop)
            if causal:
                mask = offs[None, :] <= abs_q[:, None]        # (seq_q, n)
                s = np.where(mask[None], s, F32(-np.inf))
            block_max = s.max(axis=2)
            new_max = np.maximum(row_max, block_max)
            rescale = np.exp(row_max - new_max).astype(F32)
            p = np.exp(s - new_max[..., None]).astype(F32)
            block_sum = p.sum(axis=2, dtype=F32)
            acc = acc * rescale[..., None] + np.einsum("hqn,hnd->hqd", p, vb,
                                                       dtype=F32)
            row_sum = row_sum * rescale + block_sum
            row_max = new_max
    return (acc / row_sum[..., None]).astype(F32).reshape(n_head * seq_q, d)


def gqa_decode(q, k_cache, v_cache, seq_lens, sm_scale=None):
    """Batched decode attention over the preallocated cache.

    q (B, H, d); caches (B, Hkv, max_seq, d); seq_lens (B,). Every sequence is
    independent (the reference is batch-1, smollm2_triton/model.py:436), so
    this is ``gqa_attention`` with seq_q = 1, causal=False per sequence, on
    the first ``seq_lens[b]`` cache rows (smollm2_triton/model.py:305-314).
    """
    q = np.asarray(q, F32)
    B, H, d = q.shape
    Hkv = k_cache.shape[1]
    out = np.zeros((B, H, d), F32)
    for b in range(B):
        L = int(seq_lens[b])
        if L <= 0:
            continue
        kf = np.asarray(k_cache[b, :, :L], F32).reshape(-1, d)
        vf = np.asarray(v_cache[b, :, :L], F32).reshape(-1, d)
        out[b] = gqa_attention(q[b], kf, vf, H, Hkv, causal=False,
                               sm_scale=sm_scale)
    return out


# ---------------------------------------------------------------- norms ----
def rms_norm(x, w, eps=1e-5):
    """triton_llm/kernels/rms_norm.py:50-55: y = (x / sqrt(sum(x^2)/N + eps)) * w."""
    x = np.asarray(x, F32)
    n = x.shape[-1]
    ss = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    rms = np.sqrt(ss / F32(n) + F32(eps)).astype(F32)
    return ((x / rms) * np.asarray(w, F32)).astype(F32)


def layer_norm(x, gamma, beta, eps=1e-5):
    """triton_llm/kernels/layernorm.py:56-66 (two-pass mean / variance)."""
    x = np.asarray(x, F32)
    n = x.shape[-1]
    mean = np.sum(x, axis=-1, dtype=F32, keepdims=True) / F32(n)
    xc = x - mean
    var = np.sum(xc * xc, axis=-1, dtype=F32, keepdims=True) / F32(n)
    rstd = F32(1.0) / np.sqrt(var + F32(eps))
    return (xc * rstd * np.asarray(gamma, F32) + np.asarray(beta, F32)).astype(F32)


# ----------------------------------------------------------------- rope ----
def precompute_cos_sin(max_seq_len, d_k, theta=100000.0):
    """triton_llm/kernels/rope.py:110-121, fp32 table (max_seq_len, d_k//2)."""
    half = d_k // 2
    positions = np.arange(max_seq_len, dtype=F32)
    indices = np.arange(half, dtype=F32)
    freqs = 1.0 / (theta ** (2 * indices / d_k))
    angles = np.outer(positions, freqs)
    return np.cos(angles).astype(F32), np.sin(angles).astype(F32)


def apply_rope(x, cos, sin, seq_len, position_offset=0):
    """triton_llm/kernels/rope.py:49-66, rows (n_rows, d_k).

    Row r sits at position (r % seq_len) + position_offset; the pair is
    (x[i], x[i + d/2]) and each product is rounded before the add/subtract.
    """
    x = np.asarray(x, F32)
    n_rows, d = x.shape
    half = d // 2
    pos = (np.arange(n_rows) % seq_len) + position_offset
    c = cos[pos]
    s = sin[pos]
    xe, xo = x[:, :half], x[:, half:]
    out = np.empty_like(x)
    out[:, :half] = (xe * c) - (xo * s)
    out[:, half:] = (xe * s) + (xo * c)
    return out


def rope_positions(x, cos, sin, positions):
    """Same rotation with an explicit position per row."""
    x = np.asarray(x, F32)
    half = x.shape[-1] // 2
    c = cos[positions]
    s = sin[positions]
    xe, xo = x[..., :half], x[..., half:]
    out = np.empty_like(x)
    out[..., :half] = (xe * c) - (xo * s)
    out[..., half:] = (xe * s) + (xo * c)
    return out


# ---------------------------------------------------------- activations ----
def swiglu(gate, up):
    """triton_llm/kernels/swiglu.py:51-56 (abs-based single-exp sigmoid)."""
    x = np.asarray(gate, F32)
    y = np.asarray(up, F32)
    e = np.exp(-np.abs(x)).astype(F32)
    one = F32(1.0)
    sig = np.where(x >= 0, one / (one + e), e / (one + e)).astype(F32)
    return ((x * sig) * y).astype(F32)


def gelu(x):
    """triton_llm/kernels/gelu.py:17-28 and :50-51 (tanh built from exp)."""
    x = np.asarray(x, F32)
    u = F32(0.7978845608028654) * (x + F32(0.044715) * x * x * x)
    e = np.exp(F32(-2.0) * np.abs(u)).astype(F32)
    sign = np.where(u < 0, F32(-1.0), F32(1.0))
    t = sign * (F32(1.0) - e) / (F32(1.0) + e)
    return (F32(0.5) * x * (F32(1.0) + t)).astype(F32)


def add(x, y):
    """triton_llm/kernels/add.py:49-51."""
    return (np.asarray(x, F32) + np.asarray(y, F32)).astype(F32)


def embedding(token_ids, wte, wpe, position_offset=0):
    """triton_llm/kernels/embedding.py:75-94: wte[id] + wpe[s + offset]."""
    ids = np.asarray(token_ids)
    b, s = ids.shape
    pos = np.arange(s) + position_offset
    return (np.asarray(wte, F32)[ids] + np.asarray(wpe, F32)[pos][None]).astype(F32)


def gemm(a, b):
    """triton_llm/kernels/gemm.py:40-48 in fp32 (the interpreter's tl.dot)."""
    return np.matmul(np.asarray(a, F32), np.asarray(b, F32)).astype(F32)


def softmax(x):
    """Row softmax (triton_llm/kernels/softmax.py), max-subtracted, fp32."""
    x = np.asarray(x, F32)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m).astype(F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)


def argmax(logits):
    """Greedy sampling: first maximal index (smollm2_triton/model.py:583)."""
    return np.argmax(np.asarray(logits), axis=-1)


def sample(logits, temperature, top_k, u):
    """Temperature / top-k sampling (smollm2_triton/model.py:566-582) with
    the uniform ``u`` that np.random.choice would draw.

    Restates the reference's arithmetic: scaled = logits / T in float32,
    probs = exp(scaled - max) in float32 widened to float64 and normalised;
    with 0 < top_k the top_k largest probabilities are kept and renormalised
    (np.argpartition). Here they are the top_k largest logits, which are top_k
    largest probabilities because exp(x / T - max) does not decrease in x;
    among equal logits the lowest indices are kept (the reference leaves the
    choice among equal probabilities open). Then NumPy's
    choice(V, p=probs): cdf = cumsum(p); cdf /= cdf[-1]; the sample is
    cdf.searchsorted(u, side='right'), the first index whose cdf exceeds u.
    ``temperature`` must be > 1e-6 (the reference takes argmax below that).
    """
    return int(sample_cdf(logits, temperature, top_k).searchsorted(float(u), side="right"))


def sample_cdf(logits, temperature, top_k):
    """The normalised cdf ``sample`` searches (for boundary-distance checks)."""
    x = np.asarray(logits, F32).reshape(-1)
    scaled = (x / F32(temperature)).astype(F32)
    probs = np.exp(scaled - np.max(scaled)).astype(np.float64)
    probs = probs / np.sum(probs)
    if top_k > 0:
        k = min(int(top_k), len(probs))
        order = np.argsort(-x, kind="stable")[:k]
        filtered = np.zeros_like(probs)
        filtered[order] = probs[order]
        probs = filtered / filtered.sum()
    cdf = np.cumsum(probs)
    return cdf / cdf[-1]
