"""Numpy restatement of the reference models' cached forward passes.

Test infrastructure only. ``SmolLM2Oracle`` follows
smollm2_triton/model.py:51-140 (weight layout) and :231-379 (prefill and
decode through the preallocated cache); ``GPT2Oracle`` follows
gpt2_triton/model.py:53-176 and :275-368.

Storage precision is a parameter so the same restatement checks both modes
of the B200 path:

* ``weight_dtype="float32"``: the reference exactly (fp32 everything);
* ``weight_dtype="bfloat16"``: every Linear weight and the embedding table
  are rounded to bf16 once at load; K and V are rounded to bf16 when they
  are appended to the cache, and attention reads the rounded values (both
  for decode and prefill). Activations, norms, attention outputs and logits
  stay fp32 -- the storage points of the B200 bf16 path.
* ``act_dtype="bfloat16"`` (SmolLM2 only) additionally rounds every
  projection input to bf16 where the B200 path stores it as a one-plane
  bf16 operand: the attention output, the SwiGLU output and the inputs of
  the projections after each RMSNorm. The B200 path folds most RMSNorms
  into the projections around them (the norm weight on the operand, the
  row's 1/rms after the product): there the stored operand is h * w and
  the product is divided by the rms afterwards -- ln2 of every layer, ln1
  of every layer but the first, and the final norm of single-token steps.
  The first layer's ln1 and a prefill's final norm round the normalised
  rows themselves. The residual stream, q and the logits stay fp32.
"""

from __future__ import annotations

import numpy as np

from . import ops

F32 = np.float32


def _store(x, bf16):
    return ops.bf16_round(x) if bf16 else np.asarray(x, F32)


def _rms(h, eps):
    """The rms of each row as ops.rms_norm computes it."""
    h = np.asarray(h, F32)
    ss = np.sum(h * h, axis=-1, dtype=F32, keepdims=True)
    return np.sqrt(ss / F32(h.shape[-1]) + F32(eps)).astype(F32)


class SmolLM2Oracle:
    """One sequence of a SmolLM2 / Llama model (batch 1, like the reference)."""

    def __init__(self, config, weights, weight_dtype="float32",
                 kv_dtype=None, act_dtype="float32"):
        self.config = c = config
        self.wbf16 = weight_dtype in ("bfloat16", "bf16")
        kvd = kv_dtype or weight_dtype
        self.kvbf16 = kvd in ("bfloat16", "bf16")
        self.actbf16 = act_dtype in ("bfloat16", "bf16")
        wb = self.wbf16
        self.n_layer = c.num_hidden_layers
        self.H = c.num_attention_heads
        self.Hkv = c.num_key_value_heads
        self.d = c.hidden_size // self.H
        self.eps = c.rms_norm_eps
        # smollm2_triton/model.py:52-76: embedding, final norm, tied lm_head
        self.wte = _store(weights["model.embed_tokens.weight"], wb)
        self.ln_f = np.asarray(weights["model.norm.weight"], F32)
        if "lm_head.weight" in weights:
            lm = _store(weights["lm_head.weight"], wb)
        else:
            lm = self.wte
        self.lm_head_w = np.ascontiguousarray(lm.T)           # (hidden, vocab)
        # :89-140: Linear weights transposed to (in, out)
        L = []
        for i in range(self.n_layer):
            p = f"model.layers.{i}."
            L.append(dict(
                wq=_store(weights[p + "self_attn.q_proj.weight"], wb).T.copy(),
                wk=_store(weights[p + "self_attn.k_proj.weight"], wb).T.copy(),
                wv=_store(weights[p + "self_attn.v_proj.weight"], wb).T.copy(),
                wo=_store(weights[p + "self_attn.o_proj.weight"], wb).T.copy(),
                wg=_store(weights[p + "mlp.gate_proj.weight"], wb).T.copy(),
                wu=_store(weights[p + "mlp.up_proj.weight"], wb).T.copy(),
                wd=_store(weights[p + "mlp.down_proj.weight"], wb).T.copy(),
                ln1=np.asarray(weights[p + "input_layernorm.weight"], F32),
                ln2=np.asarray(weights[p + "post_attention_layernorm.weight"], F32),
            ))
        self.layers = L
        self.cos, self.sin = ops.precompute_cos_sin(
            c.max_position_embeddings, self.d, c.rope_theta)
        self.cache = None
        self.cache_len = 0

    # smollm2_triton/model.py:190-225
    def init_cache(self, max_seq=None):
        max_seq = max_seq or self.config.max_position_embeddings
        self.cache = [dict(k=np.zeros((self.Hkv, max_seq, self.d), F32),
                           v=np.zeros((self.Hkv, max_seq, self.d), F32))
                      for _ in range(self.n_layer)]
        self.cache_len = 0

    def forward_cached(self, token_ids):
        """smollm2_triton/model.py:231-379 -> logits (1, seq, vocab)."""
        ids = np.asarray(token_ids).reshape(1, -1)
        seq = ids.shape[1]
        H, Hkv, d = self.H, self.Hkv, self.d
        prev = self.cache_len
        total = prev + seq
        h = self.wte[ids[0]].astype(F32)                      # (seq, hidden)
        for i, Lw in enumerate(self.layers):
            cache = self.cache[i]
            residual = h
            q, k, v = self._normed_gemms(h, Lw["ln1"], (Lw["wq"], Lw["wk"], Lw["wv"]),
                                         folded=i > 0)
            qh = q.reshape(seq, H, d).transpose(1, 0, 2).reshape(-1, d)
            kh = k.reshape(seq, Hkv, d).transpose(1, 0, 2).reshape(-1, d)
            vh = v.reshape(seq, Hkv, d).transpose(1, 0, 2).reshape(-1, d)
            qh = ops.apply_rope(qh, self.cos, self.sin, seq, prev)
            kh = ops.apply_rope(kh, self.cos, self.sin, seq, prev)
            cache["k"][:, prev:total] = _store(kh.reshape(Hkv, seq, d), self.kvbf16)
            cache["v"][:, prev:total] = _store(vh.reshape(Hkv, seq, d), self.kvbf16)
            if seq == 1:
                kf = cache["k"][:, :total].reshape(-1, d)
                vf = cache["v"][:, :total].reshape(-1, d)
                o = ops.gqa_attention(qh, kf, vf, H, Hkv, causal=False)
            else:
                if self.kvbf16:
                    kf = cache["k"][:, prev:total].reshape(-1, d)
                    vf = cache["v"][:, prev:total].reshape(-1, d)
                else:
                    kf, vf = kh, vh
                o = ops.gqa_attention(qh, kf, vf, H, Hkv, causal=True)
            o = o.reshape(H, seq, d).transpose(1, 0, 2).reshape(seq, H * d)
            o = _store(o, self.actbf16)
            h = ops.add(ops.gemm(o, Lw["wo"]), residual)
            residual = h
            g, u = self._normed_gemms(h, Lw["ln2"], (Lw["wg"], Lw["wu"]), folded=True)
            act = _store(ops.swiglu(g, u), self.actbf16)
            h = ops.add(ops.gemm(act, Lw["wd"]), residual)
        self.cache_len = total
        (logits,) = self._normed_gemms(h, self.ln_f, (self.lm_head_w,), folded=seq == 1)
        return logits.reshape(1, seq, -1)

    def _normed_gemms(self, h, w_norm, mats, folded):
        """rms_norm(h) @ each matrix (smollm2_triton/model.py:281-287, :357-365,
        :371-375). With bf16 projection inputs, a norm the B200 path folds
        stores h * w (rounded) and divides the products by the rms."""
        if self.actbf16 and folded:
            xw = _store(np.asarray(h, F32) * np.asarray(w_norm, F32), True)
            rms = _rms(h, self.eps)
            return [(ops.gemm(xw, m) / rms).astype(F32) for m in mats]
        x = _store(ops.rms_norm(h, w_norm, self.eps), self.actbf16)
        return [ops.gemm(x, m) for m in mats]

    def generate(self, token_ids, max_new_tokens, max_seq=None):
        """Greedy generation (smollm2_triton/model.py:452-469), returns ids
        and the logits of every step."""
        ids = np.asarray(token_ids, np.int32).reshape(1, -1)
        self.init_cache(max_seq or ids.shape[1] + max_new_tokens)
        logits = self.forward_cached(ids)
        out = list(ids[0])
        all_logits = []
        for step in range(max_new_tokens):
            last = logits[0, -1]
            all_logits.append(last.copy())
            tok = int(ops.argmax(last))
            out.append(tok)
            if step < max_new_tokens - 1:
                logits = self.forward_cached(np.array([[tok]], np.int32))
        return np.array([out], np.int32), np.stack(all_logits)


class GPT2Oracle:
    """GPT-2 with a preallocated fp32 cache (gpt2_triton/model.py:275-368)."""

    def __init__(self, config, weights):
        self.config = c = config
        self.H = c.n_head
        self.d = c.n_embd // c.n_head
        self.eps = c.layer_norm_epsilon
        g = lambda k: np.asarray(weights[k], F32)  # noqa: E731
        self.wte, self.wpe = g("wte.weight"), g("wpe.weight")
        self.lm_head_w = np.ascontiguousarray(self.wte.T)
        self.ln_f = (g("ln_f.weight"), g("ln_f.bias"))
        self.layers = []
        for i in range(c.n_layer):
            p = f"h.{i}."
            self.layers.append(dict(
                ln1=(g(p + "ln_1.weight"), g(p + "ln_1.bias")),
                ln2=(g(p + "ln_2.weight"), g(p + "ln_2.bias")),
                w_attn=g(p + "attn.c_attn.weight"), b_attn=g(p + "attn.c_attn.bias"),
                w_proj=g(p + "attn.c_proj.weight"), b_proj=g(p + "attn.c_proj.bias"),
                w_fc=g(p + "mlp.c_fc.weight"), b_fc=g(p + "mlp.c_fc.bias"),
                w_mproj=g(p + "mlp.c_proj.weight"), b_mproj=g(p + "mlp.c_proj.bias"),
            ))
        self.cache = None
        self.cache_len = 0

    def init_cache(self, max_seq=None):
        max_seq = max_seq or self.config.n_positions
        self.cache = [dict(k=np.zeros((self.H, max_seq, self.d), F32),
                           v=np.zeros((self.H, max_seq, self.d), F32))
                      for _ in self.layers]
        self.cache_len = 0

    def forward_cached(self, token_ids):
        ids = np.asarray(token_ids).reshape(1, -1)
        seq = ids.shape[1]
        H, d = self.H, self.d
        n = H * d
        prev = self.cache_len
        total = prev + seq
        h = ops.embedding(ids, self.wte, self.wpe, prev).reshape(seq, n)
        for i, Lw in enumerate(self.layers):
            residual = h
            x = ops.layer_norm(h, *Lw["ln1"], self.eps)
            qkv = ops.add(ops.gemm(x, Lw["w_attn"]), Lw["b_attn"])
            q, k, v = qkv[:, :n], qkv[:, n:2 * n], qkv[:, 2 * n:]
            c = self.cache[i]
            c["k"][:, prev:total] = k.reshape(seq, H, d).transpose(1, 0, 2)
            c["v"][:, prev:total] = v.reshape(seq, H, d).transpose(1, 0, 2)
            qh = q.reshape(seq, H, d).transpose(1, 0, 2).reshape(-1, d)
            kf = c["k"][:, :total].reshape(-1, d)
            vf = c["v"][:, :total].reshape(-1, d)
            if seq == 1:
                o = ops.gqa_attention(qh, kf, vf, H, H, causal=False)
            else:
                # prefill starts from an empty cache: seq_k == seq_q
                o = ops.gqa_attention(qh, kf, vf, H, H, causal=True)
            o = o.reshape(H, seq, d).transpose(1, 0, 2).reshape(seq, n)
            out = ops.add(ops.gemm(o, Lw["w_proj"]), Lw["b_proj"])
            h = ops.add(out, residual)
            residual = h
            x = ops.layer_norm(h, *Lw["ln2"], self.eps)
            m = ops.gelu(ops.add(ops.gemm(x, Lw["w_fc"]), Lw["b_fc"]))
            m = ops.add(ops.gemm(m, Lw["w_mproj"]), Lw["b_mproj"])
            h = ops.add(m, residual)
        self.cache_len = total
        x = ops.layer_norm(h, *self.ln_f, self.eps)
        return ops.gemm(x, self.lm_head_w).reshape(1, seq, -1)

    def generate(self, token_ids, max_new_tokens, max_seq=None):
        ids = np.asarray(token_ids, np.int32).reshape(1, -1)
        self.init_cache(max_seq or ids.shape[1] + max_new_tokens)
        logits = self.forward_cached(ids)
        out = list(ids[0])
        all_logits = []
        for step in range(max_new_tokens):
            last = logits[0, -1]
            all_logits.append(last.copy())
            tok = int(ops.argmax(last))
            out.append(tok)
            if step < max_new_tokens - 1:
                logits = self.forward_cached(np.array([[tok]], np.int32))
        return np.array([out], np.int32), np.stack(all_logits)
