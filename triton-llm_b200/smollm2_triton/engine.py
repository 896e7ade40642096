"""Batched decode engine for SmolLM2 / Llama models on sm_100a.

The math is the reference's cached forward pass
(smollm2_triton/model.py:231-379) for B independent sequences at once:

  h = embed(ids)                                        model.py:271, 547-560
  per layer:
    x = rmsnorm(h) ; q, k, v = x Wq, x Wk, x Wv         model.py:281-287
    rope(q), rope(k) ; cache[pos] = k, v                model.py:296-302
    o = gqa_attention(q, cache[:len])                   model.py:305-314
    h = h + o Wo                                        model.py:351-353
    x = rmsnorm(h) ; h = h + swiglu(x Wg, x Wu) Wd      model.py:357-365
  logits = rmsnorm(h) W_lm                              model.py:371-375

mapped onto seven kernels per layer: RMSNorm, the QKV projection with RoPE
and the KV-cache append in its epilogue, split-KV attention, the o
projection with the residual add in its epilogue, RMSNorm, the gate/up
projection with SwiGLU in its epilogue, and the down projection with the
residual add. Token ids, positions and lengths live on the device and greedy
sampling is an on-device argmax, so a decode step has no host round trip and
can be captured as one CUDA graph.

KV cache layout: per layer k and v (B, n_kv_head, max_seq, head_dim), the
reference's (n_kv_head, max_seq, d_k) (model.py:219-225) with a batch axis.

Activation buffers that only feed projections (the normed x, the attention
output, the SwiGLU output) are kept in the tensor-core operand format when
the weights are bf16 -- hi + lo bf16 planes (act_dtype="split", the
default: ~16 mantissa bits, close to the reference's fp32 activations) or
one bf16 plane (act_dtype="bfloat16") -- and the kernels that produce them
write that format directly. The residual stream h, q and the logits stay
fp32.
"""

from __future__ import annotations

import os

import numpy as np

from triton_llm import gpu, _lib, shard
from triton_llm.kernels import gqa_rows, gqa_prefill, prefill_blocks, DecodeWorkspace
from triton_llm.kernels.attention_prefill import prefill_supported
from triton_llm.kernels.linear import (FoldedNorm, Linear, LinearWorkspace, kernel_name,
                                       linear, qkv_rows, swiglu_rows)
from triton_llm.kernels.rms_norm import (rms_norm_add_rows, rms_norm_p2p_rows,
                                         rms_norm_rows)
from triton_llm.kernels.rope import precompute_cos_sin
from triton_llm.kernels.embedding import embedding_dev
from triton_llm.kernels import mlp as _mlp
from triton_llm.tp import PeerGroup


def _dtype_of(config, dtype):
    d = dtype or getattr(config, "torch_dtype", "float32") or "float32"
    return "bfloat16" if d in ("bfloat16", "bf16") else "float32"


class LlamaWeights:
    """All weights of a Llama-family model on the device, in kernel layout."""

    def __init__(self, config, weights=None, dtype=None, seed=None, std=0.02,
                 max_pos=None, tp_rank=0, tp_size=1):
        c = self.config = config
        self.dtype = _dtype_of(config, dtype)
        self.bf16 = self.dtype == "bfloat16"
        self.n = c.hidden_size
        self.D = self.n // c.num_attention_heads
        self.V = c.vocab_size
        self.L = c.num_hidden_layers
        self.eps = float(c.rms_norm_eps)
        if c.num_attention_heads % c.num_key_value_heads:
            raise ValueError(f"n_head ({c.num_attention_heads}) must be divisible by "
                             f"n_kv_head ({c.num_key_value_heads})")
        # tensor parallelism by KV head: H, Hkv, F are this rank's shares
        self.tp_rank, self.tp_size = int(tp_rank), int(tp_size)
        self.H, self.Hkv, self.F = shard.tp_dims(
            c.num_attention_heads, c.num_key_value_heads, c.intermediate_size,
            self.tp_size)
        self.max_pos = int(max_pos or c.max_position_embeddings)
        cos, sin = precompute_cos_sin(self.max_pos, self.D, c.rope_theta)
        self.cos, self.sin = gpu.to_device(cos), gpu.to_device(sin)
        if weights is not None:
            self._from_state_dict(weights)
        else:
            self._random(seed if seed is not None else 0, std)

    # -- from a HF-style state dict (numpy arrays, (out, in) Linear layout)
    def _from_state_dict(self, w):
        dt = self.dtype
        f32 = lambda a: gpu.to_device(np.ascontiguousarray(a, np.float32))  # noqa: E731
        c = self.config
        self.layers = []
        for i in range(self.L):
            lw = shard.shard_llama_layer(w, f"model.layers.{i}.", self.D,
                                         c.num_attention_heads, c.num_key_value_heads,
                                         c.intermediate_size, self.tp_rank, self.tp_size)
            wqkv, _ = qkv_rows(lw["q"], lw["k"], lw["v"], self.D)
            self.layers.append(dict(
                qkv=Linear(wqkv, dt),
                o=Linear(lw["o"], dt),
                gu=Linear(swiglu_rows(np.asarray(lw["gate"], np.float32),
                                      np.asarray(lw["up"], np.float32)), dt),
                down=Linear(lw["down"], dt),
                ln1=f32(lw["ln1"]),
                ln2=f32(lw["ln2"]),
            ))
        self.norm = f32(w["model.norm.weight"])
        emb = w["model.embed_tokens.weight"]
        self.lm_head = Linear(w["lm_head.weight"] if "lm_head.weight" in w else emb, dt)
        if "lm_head.weight" in w:
            self.embed = Linear(emb, dt)
        else:
            if not getattr(self.config, "tie_word_embeddings", True):
                raise KeyError("lm_head.weight is missing from weights and "
                               "tie_word_embeddings is False")
            self.embed = self.lm_head          # tied: one device copy

    # -- random-init N(0, std) on the device (benchmarks)
    def _random(self, seed, std):
        dt = _lib.BF16 if self.bf16 else _lib.F32
        counter = [seed * 1000003]

        def rnd(shape, s=std):
            t = gpu.allocate(shape, "bfloat16" if self.bf16 else np.float32)
            counter[0] += 1
            _lib.call("tllm_fill_random", t.ptr, dt, int(np.prod(shape)),
                      counter[0], float(s), None)
            return t

        def lin(N, K):
            if self.bf16:
                obj = Linear.empty_bf16(N, K)
                counter[0] += 1
                _lib.call("tllm_fill_random", obj.w.ptr, _lib.BF16,
                          int(obj.w.shape[0]), counter[0], float(std), None)
                return obj
            obj = Linear.__new__(Linear)
            obj.N, obj.K, obj.bf16, obj.b = N, K, False, None
            obj.w = rnd((N, K))
            return obj

        def norm_w():
            t = gpu.allocate((self.n,), np.float32)
            counter[0] += 1
            _lib.call("tllm_fill_random", t.ptr, _lib.F32, self.n, counter[0],
                      float(std), None)
            return t

        n, D = self.n, self.D
        self.layers = []
        for _ in range(self.L):
            self.layers.append(dict(qkv=lin((self.H + 2 * self.Hkv) * D, n),
                                    o=lin(n, self.H * D), gu=lin(2 * self.F, n),
                                    down=lin(n, self.F), ln1=norm_w(), ln2=norm_w()))
        self.norm = norm_w()
        self.lm_head = lin(self.V, n)
        self.embed = self.lm_head

    def linear_shapes(self, M):
        n, D = self.n, self.D
        return [(M, (self.H + 2 * self.Hkv) * D, n), (M, n, self.H * D),
                (M, 2 * self.F, n), (M, n, self.F), (M, self.V, n)]

    def nbytes(self):
        per = 2 if self.bf16 else 4
        n, D = self.n, self.D
        layer = ((self.H + 2 * self.Hkv) * D * n + n * self.H * D + 2 * self.F * n
                 + n * self.F) * per + 2 * n * 4
        return self.L * layer + self.V * n * per + n * 4


class LlamaSession:
    """KV caches and step buffers for ``batch`` sequences of a model."""

    def __init__(self, wts: LlamaWeights, batch: int, max_seq: int,
                 max_prefill_rows: int = 0, attn_budget_bytes: int = 256 << 20,
                 kv_dtype: str | None = None, act_dtype: str = "split",
                 tp=None, p2p: bool | None = None):
        self.w = wts
        # tensor parallelism: o / down produce partial sums that ``tp``
        # (a triton_llm.tp.TPGroup) all-reduces; the residual add moves into
        # the next RMSNorm. Decode rows reduce through the fused peer-to-peer
        # path (p2p=True, the default; TLLM_TP_P2P=0 turns it off), prefill
        # rows through NCCL.
        self.tp = tp
        if p2p is None:
            p2p = os.environ.get("TLLM_TP_P2P", "1") != "0"
        tp_size = tp.size if tp is not None else 1
        if tp_size != wts.tp_size:
            raise ValueError(f"weights are sharded {wts.tp_size}-way, group has {tp_size}")
        # projection inputs: "bfloat16" (one bf16 plane) or "split" (bf16
        # hi + lo, ~16 mantissa bits); fp32 weights take fp32 activations
        if act_dtype not in ("bfloat16", "bf16", "split"):
            raise ValueError(f"act_dtype must be 'bfloat16' or 'split', got {act_dtype!r}")
        self.act_planes = 2 if act_dtype == "split" else 1
        self.B = int(batch)
        self.S = int(max_seq)
        if self.S > wts.max_pos:
            raise ValueError(f"max_seq ({self.S}) exceeds the RoPE table "
                             f"({wts.max_pos} positions)")
        B, S, Hkv, D = self.B, self.S, wts.Hkv, wts.D
        # KV cache precision follows the weights unless given ("float32" keeps
        # the reference's fp32 cache under bf16 weights)
        self.kv_bf16 = wts.bf16 if kv_dtype is None else kv_dtype in ("bfloat16", "bf16")
        kvdt = "bfloat16" if self.kv_bf16 else np.float32
        per_layer = 2 * B * Hkv * S * D
        self.kv_arena = gpu.zeros((wts.L * per_layer,), kvdt)
        esz = 2 if self.kv_bf16 else 4
        self.kv = []
        for i in range(wts.L):
            k = gpu.sub_view(self.kv_arena, (2 * i) * (per_layer // 2) * esz,
                             (B, Hkv, S, D))
            v = gpu.sub_view(self.kv_arena, (2 * i + 1) * (per_layer // 2) * esz,
                             (B, Hkv, S, D))
            self.kv.append((k, v))
        self.pos = gpu.zeros((B,), np.int32)     # next position of each sequence
        self.lens = gpu.zeros((B,), np.int32)    # keys attended in the current step
        self.ids = gpu.zeros((B,), np.int32)     # tokens fed to the next step
        self.u = gpu.zeros((B,), np.float64)     # uniforms of a sampled step
        self.row_seq = gpu.to_device(np.arange(B, dtype=np.int32))
        self._p2p = bool(p2p)
        self._buffers(B)
        self.attn_ws = DecodeWorkspace(B, wts.H, Hkv, D, S,
                                       _lib.BF16 if self.kv_bf16 else _lib.F32)
        self.lin_ws = LinearWorkspace(wts.linear_shapes(B))
        self._prefill_rows = 0
        self._p_blocks, self._p_nblocks = None, 0
        if max_prefill_rows:
            self._prefill_buffers(max_prefill_rows, attn_budget_bytes)
        self.graph = None
        # keys a decode step's attention reads in all (sum of pos + 1), as
        # last known on the host: plans the split-KV sizes of small batches
        # (tllm_gqa_rows_hint); 0 = unknown
        self._keys_hint = 0

    def _act(self, rows, cols):
        """A projection-input buffer: bf16 operand format for bf16 weights,
        else fp32."""
        if self.w.bf16:
            return gpu.act_empty(rows, cols, self.act_planes)
        return gpu.allocate((rows, cols), np.float32)

    def _buffers(self, M):
        w = self.w
        f = lambda *s: gpu.allocate(s, np.float32)  # noqa: E731
        self.h, self.x = f(M, w.n), self._act(M, w.n)
        self.q, self.attn = f(M, w.H, w.D), self._act(M, w.H * w.D)
        self.act, self.logits = self._act(M, w.F), f(M, w.V)
        self.part = f(M, w.n) if self.tp is not None and self.tp.size > 1 else None
        # RMSNorms folded into the projections around them (bf16 weights,
        # unsharded layers, every projection on the tensor-core kernel, whose
        # idle warps sum the producer's partials during the weight stream; the
        # skinny kernel would wait for those loads on its critical path):
        # partial sums of squares of h per column part
        self._fold_ok = (w.bf16 and self.part is None
                         and os.environ.get("TLLM_NORM_FOLD", "1") != "0")
        self.ss = (f(-(-w.n // 16), M) if self._fold_ok and self._all_tensor_core(M)
                   else None)
        self.peer = None
        if self.part is not None and self._p2p:
            self.peer = self.tp.peer_group(M, w.n)
        # decode rows: o, norm, gate/up and down in one launch (tllm_mlp,
        # TLLM_FUSED_MLP=1) for bf16 weights, one-plane operands and shapes it
        # covers. Off by default: at config 4 it measures 87 us per layer
        # against 52 us for the four launches, its split-K epilogues being
        # slower than the clusters' distributed-shared-memory reduction.
        self.mlp_ws = None
        if (os.environ.get("TLLM_FUSED_MLP", "0") == "1" and self.part is None
                and w.bf16 and self.act_planes == 1 and w.n >= 1024
                and _mlp.supported(M, w.H * w.D, w.n, w.F)
                and all(w.layers[0][k].tiled for k in ("o", "gu", "down"))):
            self.mlp_ws = _mlp.MlpWorkspace(M, w.H * w.D, w.n, w.F)

    def _all_tensor_core(self, M):
        """Whether every projection of a layer (and the lm_head) runs on the
        tcgen05 kernel for M rows."""
        return all(kernel_name(m, n, k) == "linear_tc_kernel"
                   for (m, n, k) in self.w.linear_shapes(M))

    def _prefill_buffers(self, M, attn_budget):
        w = self.w
        f = lambda *s: gpu.allocate(s, np.float32)  # noqa: E731
        self.p_h, self.p_x = f(M, w.n), self._act(M, w.n)
        self.p_q, self.p_attn = f(M, w.H, w.D), self._act(M, w.H * w.D)
        self.p_act = self._act(M, w.F)
        self.p_part = f(M, w.n) if self.part is not None else None
        self.p_ss = (f(-(-w.n // 16), M) if self._fold_ok and self._all_tensor_core(M)
                     else None)
        self.p_ids = gpu.allocate((M,), np.int32)
        self.p_seq = gpu.allocate((M,), np.int32)
        self.p_pos = gpu.allocate((M,), np.int32)
        self.p_len = gpu.allocate((M,), np.int32)
        self.p_last = gpu.allocate((self.B,), np.int32)
        self.p_lin_ws = LinearWorkspace(w.linear_shapes(M))
        ws = DecodeWorkspace.__new__(DecodeWorkspace)
        ws.partial_bytes = int(attn_budget)
        ws.partial = gpu.allocate((max(attn_budget // 4, 1),), np.float32)
        ws.counters = gpu.zeros((M * w.H,), np.int32)
        self.p_attn_ws = ws
        self._prefill_rows = M

    # ------------------------------------------------------------------
    def _layer(self, i, M, h, x, q, attn, act, row_seq, row_pos, lens, ws,
               decode, attn_ws, row_len=None, max_len=None, part=None):
        """One layer on rows 0..M-1. With tensor parallelism (``part`` set)
        o / down write partial sums into ``part``, which is all-reduced and
        added to h by the next RMSNorm (this layer's second one, the next
        layer's first, or the final norm)."""
        w = self.w
        L = w.layers[i]
        k, v = self.kv[i]
        ss = self.ss if decode else self.p_ss
        fold_ln1 = None
        if part is not None and i > 0:
            self._norm_add(h, part, L["ln1"], x, M)
        elif ss is not None and part is None and i > 0 and self.mlp_ws is None:
            # ln1 folded: the previous layer's down projection wrote h * ln1
            # and the partial sums; the QKV epilogue divides by the rms
            fold_ln1 = FoldedNorm(L["ln1"], x, ss, w.n, w.eps, M, w.F)
        else:
            rms_norm_rows(h, L["ln1"], x, M, w.eps)
        linear(x, L["qkv"], op=_lib.EPI_QKV, ws=ws, M=M, fold_in=fold_ln1, qkv=dict(
            cos=w.cos, sin=w.sin, row_seq=row_seq, row_pos=row_pos, q_out=q,
            k_cache=k, v_cache=v, n_head=w.H, n_kv_head=w.Hkv, head_dim=w.D,
            lens_out=lens if decode else None))
        # decode: row b reads its own sequence for lens[b] keys (set by the
        # QKV epilogue); prefill: row r reads its sequence's causal prefix,
        # in blocks of 64 rows (tllm_gqa_prefill) where the cache allows
        if not decode and self._p_blocks is not None:
            gqa_prefill(q, k, v, self._p_blocks, self._p_nblocks, attn, w.H,
                        w.H * w.D, w.D, w.H * w.D, w.D)
        else:
            gqa_rows(q, k, v, row_seq, lens if decode else row_len, attn, M, w.H,
                     w.H * w.D, w.D, w.H * w.D, w.D,
                     self.S if decode else (max_len or self.S), workspace=attn_ws,
                     keys_hint=self._keys_hint if decode else 0)
        if part is None and decode and self.mlp_ws is not None:
            _mlp.mlp_block(attn, L["o"], h, L["ln2"], x, L["gu"], act, L["down"], M,
                           w.eps, self.mlp_ws)
            return
        ss = self.ss if decode else self.p_ss
        if part is None and ss is not None:
            # ln2 folded: o writes h * ln2 and the partial sums, gate/up
            # divides its rows by the rms; down does the same for the next
            # norm (the next layer's ln1, or the final norm of a decode step)
            ln2 = FoldedNorm(L["ln2"], x, ss, w.n, w.eps, M, w.H * w.D)
            linear(attn, L["o"], out_dev=h, op=_lib.EPI_RESID, resid_dev=h, ws=ws, M=M,
                   fold_out=ln2)
            linear(x, L["gu"], out_dev=act, op=_lib.EPI_SWIGLU, ws=ws, M=M, fold_in=ln2)
            nxt = self._next_norm(i, x, ss, decode, M)
            linear(act, L["down"], out_dev=h, op=_lib.EPI_RESID, resid_dev=h, ws=ws, M=M,
                   fold_out=nxt)
            return
        if part is None:
            linear(attn, L["o"], out_dev=h, op=_lib.EPI_RESID, resid_dev=h, ws=ws, M=M)
            rms_norm_rows(h, L["ln2"], x, M, w.eps)
        else:
            self._reduce(attn, L["o"], part, M, ws)
            self._norm_add(h, part, L["ln2"], x, M)
        linear(x, L["gu"], out_dev=act, op=_lib.EPI_SWIGLU, ws=ws, M=M)
        if part is None:
            linear(act, L["down"], out_dev=h, op=_lib.EPI_RESID, resid_dev=h, ws=ws, M=M)
        else:
            self._reduce(act, L["down"], part, M, ws)

    def _next_norm(self, i, x, ss, decode, M):
        """The folded norm after layer i's down projection: the next layer's
        ln1, or (decode) the final norm; None after a prefill's last layer
        (the prefill normalises the rows it keeps on its own)."""
        w = self.w
        if i + 1 < w.L:
            return FoldedNorm(w.layers[i + 1]["ln1"], x, ss, w.n, w.eps, M, w.F)
        return FoldedNorm(w.norm, x, ss, w.n, w.eps, M, w.F) if decode else None

    def _reduce(self, src, lin, part, M, ws):
        """A row-parallel projection whose partial sums the group adds:
        ``part`` is a PeerGroup (fused: the epilogue scatters to every rank)
        or an fp32 buffer (stored, then NCCL all-reduce)."""
        if isinstance(part, PeerGroup):
            linear(src, lin, op=_lib.EPI_SCATTER, ws=ws, M=M, p2p=part)
        else:
            linear(src, lin, out_dev=part, op=_lib.EPI_STORE, ws=ws, M=M)
            self.tp.all_reduce(self._rows_view(part, M))

    def _norm_add(self, h, part, wn, x, M):
        """h += the group's sum of the last partial rows; x = RMSNorm(h)."""
        if isinstance(part, PeerGroup):
            rms_norm_p2p_rows(h, part, wn, x, M, self.w.eps)
        else:
            rms_norm_add_rows(h, part, wn, x, M, self.w.eps)

    def close(self):
        """Release the peer group (every rank, after a barrier)."""
        if getattr(self, "peer", None) is not None:
            self.peer.close()
            self.peer = None

    def _decode_part(self):
        return self.peer if self.peer is not None else self.part

    def _rows_view(self, t, M):
        return t if int(t.shape[0]) == M else gpu.sub_view(t, 0, (M, int(t.shape[1])))

    def _final_norm(self, h, x, M, part):
        w = self.w
        if part is None:
            rms_norm_rows(h, w.norm, x, M, w.eps)
        else:
            self._norm_add(h, part, w.norm, x, M)

    def prefill(self, prompts, all_logits=False, slots=None):
        """Run the prompts through the model into cache sequences ``slots``
        (default 0..len(prompts)-1).

        Every such sequence restarts at position 0. Returns the logits of the
        last prompt token of each prompt (host, (n, V)), or of every prompt
        token when ``all_logits`` (host, (sum(len), V)). Afterwards ``ids``
        holds the greedy next token of each prompt's sequence and ``pos`` the
        prompt lengths, ready for ``decode_step``. Without ``slots`` the other
        sequences are reset to position 0; with ``slots`` they keep their
        state (a serving loop admitting requests into free slots).
        """
        w = self.w
        prompts = [np.asarray(p, np.int32).reshape(-1) for p in prompts]
        nseq = len(prompts)
        if nseq > self.B:
            raise ValueError(f"{nseq} prompts for a batch of {self.B}")
        keep = slots is not None
        slots = np.arange(nseq, dtype=np.int32) if slots is None else \
            np.asarray(slots, np.int32).reshape(-1)
        if len(slots) != nseq or (slots < 0).any() or (slots >= self.B).any() or \
                len(set(slots.tolist())) != nseq:
            raise ValueError(f"slots {slots.tolist()} do not name {nseq} distinct "
                             f"sequences of the batch of {self.B}")
        lens = np.array([len(p) for p in prompts], np.int64)
        if (lens <= 0).any():
            raise ValueError("every prompt needs at least one token")
        if lens.max() > self.S:
            raise ValueError(f"prompt of {lens.max()} tokens exceeds max_seq {self.S}")
        M = int(lens.sum())
        if M > self._prefill_rows:
            self._prefill_buffers(M, 256 << 20)
        ids = np.concatenate(prompts)
        seq = np.repeat(slots, lens)
        pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
        self.p_ids.from_numpy(np.pad(ids, (0, self._prefill_rows - M)))
        self.p_seq.from_numpy(np.pad(seq, (0, self._prefill_rows - M)))
        self.p_pos.from_numpy(np.pad(pos, (0, self._prefill_rows - M)))
        self.p_len.from_numpy(np.pad(pos + 1, (0, self._prefill_rows - M)))
        self._p_blocks, self._p_nblocks = None, 0
        if prefill_supported(self.kv[0][0]):
            blocks = prefill_blocks(lens, slots)
            self._p_blocks = gpu.to_device(blocks)
            self._p_nblocks = len(blocks)
        h, x = self.p_h, self.p_x
        embedding_dev(gpu.sub_view(self.p_ids, 0, (M,)), w.embed, h)
        for i in range(w.L):
            self._layer(i, M, h, x, self.p_q, self.p_attn, self.p_act, self.p_seq,
                        self.p_pos, None, self.p_lin_ws, False, self.p_attn_ws,
                        row_len=self.p_len, max_len=int(lens.max()), part=self.p_part)
        if self.p_part is not None:
            # complete the residual stream before it is read row by row
            _lib.call("tllm_elementwise", _lib.EL_ADD, h.ptr, self.p_part.ptr, h.ptr,
                      M * w.n, None)
        if all_logits:
            logits = gpu.allocate((M, w.V), np.float32)
            rms_norm_rows(h, w.norm, x, M, w.eps)
            linear(x, w.lm_head, out_dev=logits, ws=self.p_lin_ws, M=M)
            host = logits.to_numpy()
            last_rows = np.cumsum(lens) - 1
            next_ids = np.argmax(host[last_rows], axis=-1).astype(np.int32)
        else:
            # last prompt row of every sequence -> the decode buffers
            last_rows = (np.cumsum(lens) - 1).astype(np.int32)
            for b, r in enumerate(last_rows):
                gpu.copy_d2d(gpu.sub_view(self.h, b * w.n * 4, (w.n,)),
                             gpu.sub_view(h, int(r) * w.n * 4, (w.n,)))
            rms_norm_rows(self.h, w.norm, self.x, nseq, w.eps)
            linear(self.x, w.lm_head, out_dev=self.logits, ws=self.lin_ws, M=nseq)
            host = self.logits.to_numpy()[:nseq]
            next_ids = np.argmax(host, axis=-1).astype(np.int32)
        if keep:
            ids_full = self.ids.to_numpy()
            pos_full = self.pos.to_numpy()
        else:
            ids_full = np.zeros(self.B, np.int32)
            pos_full = np.zeros(self.B, np.int32)
        ids_full[slots] = next_ids
        pos_full[slots] = lens
        self.ids.from_numpy(ids_full)
        self.pos.from_numpy(pos_full)
        self.lens.from_numpy(pos_full)
        self._keys_hint = int(np.sum(pos_full, dtype=np.int64)) + self.B
        return host

    def set_state(self, pos: np.ndarray, ids: np.ndarray):
        """Set positions (= cached lengths) and next tokens directly."""
        self.pos.from_numpy(np.asarray(pos, np.int32))
        self.lens.from_numpy(np.asarray(pos, np.int32))
        self.ids.from_numpy(np.asarray(ids, np.int32))
        self._keys_hint = int(np.sum(np.asarray(pos), dtype=np.int64)) + self.B

    def decode_step(self, sample=True, temperature=0.0, top_k=0):
        """One decode step for all B sequences, device only.

        Reads ``ids`` / ``pos``; leaves the step's logits in ``self.logits``
        and (sample=True) the next tokens in ``ids`` with ``pos`` advanced:
        the argmax when temperature <= 1e-6, else a temperature / top-k draw
        with the uniforms in ``self.u`` (one per sequence, set by the caller
        from the generator the reference's np.random.choice uses).
        Returns the number of kernel launches.
        """
        w = self.w
        B = self.B
        embedding_dev(self.ids, w.embed, self.h)
        for i in range(w.L):
            self._layer(i, B, self.h, self.x, self.q, self.attn, self.act,
                        self.row_seq, self.pos, self.lens, self.lin_ws, True,
                        self.attn_ws, part=self._decode_part())
        if self.ss is not None and self.mlp_ws is None:
            # the final norm folded into the lm_head (the last down projection
            # wrote h * norm and the partial sums)
            linear(self.x, w.lm_head, out_dev=self.logits, ws=self.lin_ws, M=B,
                   fold_in=FoldedNorm(w.norm, self.x, self.ss, w.n, w.eps, B, w.F))
            n = 1 + 1 + 5 * w.L + 1
        else:
            self._final_norm(self.h, self.x, B, self._decode_part())
            linear(self.x, w.lm_head, out_dev=self.logits, ws=self.lin_ws, M=B)
            n = 1 + (4 if self.mlp_ws is not None else 7) * w.L + 2
        if sample and temperature > 1e-6:
            _lib.call("tllm_sample", self.logits.ptr, B, w.V, w.V, float(temperature),
                      int(top_k), self.u.ptr, self.ids.ptr, self.pos.ptr, None)
            n += 1
        elif sample:
            _lib.call("tllm_argmax", self.logits.ptr, B, w.V, w.V, self.ids.ptr,
                      self.pos.ptr, None)
            n += 1
        return n

    def capture(self):
        """Capture one greedy decode step as a CUDA graph (self.graph)."""
        g = gpu.Graph()
        with g:
            self.decode_step(True)
        self.graph = g
        return g

    def step(self):
        """Run one decode step (the captured graph when there is one)."""
        if self.graph is not None:
            self.graph.launch()
        else:
            self.decode_step(True)

    def step_host(self, ids_in: np.ndarray | None, ids_out: np.ndarray) -> None:
        """One serving-loop step with host token buffers.

        Copies ``ids_in`` (B int32, pinned host memory, or None to keep the
        device's own next tokens) to the device, runs one greedy decode step
        (the captured graph when there is one) and copies the sampled tokens
        into ``ids_out`` (B int32, pinned), then waits for the copy.
        """
        if ids_in is not None:
            gpu.copy_h2d_async(self.ids, ids_in)
        self.step()
        gpu.copy_d2h_async(ids_out, self.ids)
        gpu.stream_synchronize()

    def kv_bytes_per_step(self, lens: np.ndarray) -> int:
        w = self.w
        return int(2 * w.L * w.Hkv * w.D * (2 if self.kv_bf16 else 4) * int(np.sum(lens)))
