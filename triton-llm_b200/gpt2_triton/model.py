"""GPT-2 model on sm_100a kernels (drop-in for gpt2_triton/model.py).

Keeps the reference's class and methods (model.py:40-554): ``forward``,
``_forward_full``, ``_init_cache``, ``_forward_cached``, ``generate``,
``generate_gpu``, ``generate_stream_gpu``, ``_sample``. Per layer
(model.py:316-361): LayerNorm, c_attn projection (+ bias) whose epilogue
writes q and appends k, v to the preallocated cache, attention over the
cache, c_proj (+ bias + residual in the epilogue), LayerNorm, c_fc (+ bias +
tanh-GELU in the epilogue), mlp c_proj (+ bias + residual). Weights stay fp32
(the reference's precision) unless ``dtype="bfloat16"``; GPT-2's Conv1D
weights, stored (in, out), are transposed once to the kernels' (out, in)
layout. The cache replaces the reference's per-head np.concatenate lists
(model.py:267-273, :340-341) with a (n_head, max_seq, d) buffer per layer.

A one-token cached forward (the decode step) replays a CUDA graph of the
whole step -- embedding to lm_head -- captured on first use: the token,
its position and the cache length reach the kernels through device
buffers, the attention's grid is sized for the full cache, so one graph
serves every position. It is captured again whenever a buffer it uses is
reallocated. ``use_graph = False`` runs the same launches one by one.
"""

from __future__ import annotations

import time

import numpy as np

from triton_llm import gpu, _lib
from triton_llm.kernels import gqa_rows, DecodeWorkspace, softmax
from triton_llm.kernels.embedding import embedding_dev
from triton_llm.kernels.layernorm import layer_norm_dev
from triton_llm.kernels.linear import Linear, LinearWorkspace, linear, qkv_rows
from .config import GPT2Config


class GPT2Model:
    """GPT-2 inference model (batch 1 API of the reference)."""

    @classmethod
    def from_safetensors(cls, path, config: GPT2Config | None = None, dtype: str = "float32"):
        """Build from a safetensors checkpoint (file, shards or directory);
        names may carry HuggingFace's ``transformer.`` prefix."""
        from collections.abc import Mapping
        from triton_llm.safetensors import load_state_dict
        sd = load_state_dict(path)
        pre = "transformer."

        class _Names(Mapping):   # lazy view without the prefix
            def __getitem__(self, k):
                return sd[k] if k in sd else sd[pre + k]

            def __iter__(self):
                return (k[len(pre):] if k.startswith(pre) else k for k in sd)

            def __len__(self):
                return len(sd)

        return cls(config or GPT2Config(), _Names(), dtype=dtype)

    def __init__(self, config: GPT2Config, weights: dict, dtype: str = "float32"):
        self.config = c = config
        self.H = c.n_head
        self.n = c.n_embd
        self.D = c.n_embd // c.n_head
        self.bf16 = dtype in ("bfloat16", "bf16")
        dt = "bfloat16" if self.bf16 else "float32"
        g = lambda k: np.asarray(weights[k], np.float32)  # noqa: E731
        f32 = lambda a: gpu.to_device(np.ascontiguousarray(a, np.float32))  # noqa: E731
        self.wte = np.require(weights["wte.weight"], np.float32, ["C_CONTIGUOUS"])
        self.wpe = np.require(weights["wpe.weight"], np.float32, ["C_CONTIGUOUS"])
        n, D = self.n, self.D
        self.layers = []
        for i in range(c.n_layer):
            p = f"h.{i}."
            wa = g(p + "attn.c_attn.weight").T          # (3n, n) = (out, in)
            ba = g(p + "attn.c_attn.bias")
            wqkv, bqkv = qkv_rows(wa[:n], wa[n:2 * n], wa[2 * n:], D,
                                  ba[:n], ba[n:2 * n], ba[2 * n:])
            self.layers.append(dict(
                ln1=(f32(g(p + "ln_1.weight")), f32(g(p + "ln_1.bias"))),
                ln2=(f32(g(p + "ln_2.weight")), f32(g(p + "ln_2.bias"))),
                qkv=Linear(wqkv, dt, bqkv),
                proj=Linear(g(p + "attn.c_proj.weight").T, dt, g(p + "attn.c_proj.bias")),
                fc=Linear(g(p + "mlp.c_fc.weight").T, dt, g(p + "mlp.c_fc.bias")),
                mproj=Linear(g(p + "mlp.c_proj.weight").T, dt, g(p + "mlp.c_proj.bias")),
            ))
        self.ln_f = (f32(g("ln_f.weight")), f32(g("ln_f.bias")))
        self.lm_head = Linear(self.wte, dt)              # tied (model.py:60-65)
        self.wte_dev = self.lm_head                      # embedding reads the same copy
        self.wpe_dev = f32(self.wpe)
        self.use_graph = True
        self._graph = None
        self._graph_key = None
        self._alloc_gen = 0   # bumped when a buffer a graph may hold is replaced
        self.kv_cache = None
        self._cache_len = 0
        self._max_seq = 0
        self._rows = 0

    # ------------------------------------------------------------------
    def _ensure_rows(self, M):
        if M <= self._rows:
            return
        c, n = self.config, self.n
        f = lambda *s: gpu.allocate(s, np.float32)  # noqa: E731
        # projection inputs in the tensor-core operand format for bf16 weights
        a = (lambda r, k: gpu.act_empty(r, k, 1)) if self.bf16 else f  # noqa: E731
        self.h, self.x = f(M, n), a(M, n)
        self.q, self.attn = f(M, self.H, self.D), a(M, n)
        self.act, self.logits = a(M, 4 * n), f(M, c.vocab_size)
        # token ids, positions and cache lengths: one buffer, one copy a step
        self.meta_d = gpu.allocate((3 * M,), np.int32)
        self.ids_d = gpu.sub_view(self.meta_d, 0, (M,))
        self.pos_d = gpu.sub_view(self.meta_d, 4 * M, (M,))
        self.len_d = gpu.sub_view(self.meta_d, 8 * M, (M,))
        self.seq_d = gpu.zeros((M,), np.int32)
        shapes = [(M, 3 * n, n), (M, n, n), (M, 4 * n, n), (M, n, 4 * n),
                  (M, c.vocab_size, n)]
        self.lin_ws = LinearWorkspace(shapes)
        self.attn_ws = None
        self._rows = M
        self._alloc_gen += 1

    def _init_cache(self, max_seq: int | None = None):
        """Empty preallocated cache (the reference starts empty lists)."""
        c = self.config
        S = int(max_seq or c.n_positions)
        if S <= 0 or S > c.n_positions:
            raise ValueError(f"max_seq must be in [1, {c.n_positions}], got {S}")
        dt = "bfloat16" if self.bf16 else np.float32
        self.kv_cache = [
            {"k": gpu.zeros((1, self.H, S, self.D), dt), "v": gpu.zeros((1, self.H, S, self.D), dt)}
            for _ in range(c.n_layer)]
        self._max_seq = S
        self._cache_len = 0
        self._alloc_gen += 1

    def _run(self, ids: np.ndarray, prev: int):
        """ids (M,) at positions prev..prev+M-1 of sequence 0 -> logits (M, V)."""
        c = self.config
        M = len(ids)
        self._ensure_rows(M)
        if (self.attn_ws is None or self.attn_ws.shape[0] < M
                or self.attn_ws.shape[4] != self._max_seq):
            kvd = _lib.BF16 if self.bf16 else _lib.F32
            self.attn_ws = DecodeWorkspace(max(M, 1), self.H, self.H, self.D,
                                           self._max_seq, kvd)
            self._alloc_gen += 1
        pos = np.arange(prev, prev + M, dtype=np.int32)
        pad = lambda a: np.pad(a, (0, self._rows - M))  # noqa: E731
        self.meta_d.from_numpy(np.concatenate([pad(ids.astype(np.int32)), pad(pos),
                                               pad(pos + 1)]))
        if M == 1 and self.use_graph:
            key = (self._rows, self._max_seq, self._alloc_gen)
            if self._graph_key != key:
                self._graph = None
                g = gpu.Graph()
                with g:
                    self._device_step(1, self._max_seq)
                self._graph, self._graph_key = g, key
            self._graph.launch()
        else:
            self._device_step(M, prev + M)
        return gpu.sub_view(self.logits, 0, (M, c.vocab_size)).to_numpy()

    def _device_step(self, M: int, max_len: int):
        """The launches of one forward over M rows (device buffers only);
        ``max_len`` bounds the cache lengths the attention grid covers."""
        c, n, H, D = self.config, self.n, self.H, self.D
        h, x = self.h, self.x
        embedding_dev(gpu.sub_view(self.ids_d, 0, (M,)), self.wte_dev, h, self.wpe_dev,
                      gpu.sub_view(self.pos_d, 0, (M,)))
        for i, L in enumerate(self.layers):
            kv = self.kv_cache[i]
            layer_norm_dev(h, L["ln1"][0], L["ln1"][1], x, c.layer_norm_epsilon, M=M)
            linear(x, L["qkv"], op=_lib.EPI_QKV, ws=self.lin_ws, M=M, qkv=dict(
                row_seq=self.seq_d, row_pos=self.pos_d, q_out=self.q,
                k_cache=kv["k"], v_cache=kv["v"], n_head=H, n_kv_head=H, head_dim=D))
            gqa_rows(self.q, kv["k"], kv["v"], self.seq_d, self.len_d, self.attn, M, H,
                     H * D, D, H * D, D, max_len, workspace=self.attn_ws)
            linear(self.attn, L["proj"], out_dev=h, op=_lib.EPI_RESID, resid_dev=h,
                   ws=self.lin_ws, M=M)
            layer_norm_dev(h, L["ln2"][0], L["ln2"][1], x, c.layer_norm_epsilon, M=M)
            linear(x, L["fc"], out_dev=self.act, op=_lib.EPI_GELU, ws=self.lin_ws, M=M)
            linear(self.act, L["mproj"], out_dev=h, op=_lib.EPI_RESID, resid_dev=h,
                   ws=self.lin_ws, M=M)
        layer_norm_dev(h, self.ln_f[0], self.ln_f[1], x, c.layer_norm_epsilon, M=M)
        linear(x, self.lm_head, out_dev=self.logits, ws=self.lin_ws, M=M)

    # ------------------------------------------------------------------
    def forward(self, token_ids: np.ndarray, use_cache: bool = False) -> np.ndarray:
        if use_cache:
            return self._forward_cached(token_ids)
        return self._forward_full(token_ids)

    def _forward_full(self, token_ids: np.ndarray) -> np.ndarray:
        """Full forward over all tokens, no cache kept (model.py:209-254)."""
        token_ids = np.asarray(token_ids)
        saved = (self.kv_cache, self._cache_len, self._max_seq)
        self._init_cache(max(token_ids.shape[1], 1))
        logits = self._run(token_ids[0], 0)
        self.kv_cache, self._cache_len, self._max_seq = saved
        self._alloc_gen += 1
        return logits.reshape(1, -1, self.config.vocab_size)

    def _forward_cached(self, token_ids: np.ndarray) -> np.ndarray:
        """Incremental forward using the cache (model.py:275-368)."""
        if self.kv_cache is None:
            raise RuntimeError("_init_cache() must be called before _forward_cached()")
        token_ids = np.asarray(token_ids)
        prev = self._cache_len
        seq = token_ids.shape[1]
        if prev + seq > self._max_seq:
            raise ValueError(f"Total sequence length {prev + seq} exceeds "
                             f"pre-allocated cache size ({self._max_seq})")
        logits = self._run(token_ids[0], prev)
        self._cache_len = prev + seq
        return logits.reshape(1, seq, self.config.vocab_size)

    # ------------------------------------------------------------------
    def _sample(self, logits: np.ndarray, temperature: float, top_k: int) -> int:
        """model.py:424-438 (softmax on the GPU for temperature sampling)."""
        if temperature > 1e-6:
            scaled = logits / temperature
            probs = softmax(scaled.reshape(1, -1)).ravel().astype(np.float64)
            if top_k > 0:
                top_k = min(top_k, len(probs))
                indices = np.argpartition(probs, -top_k)[-top_k:]
                filtered = np.zeros_like(probs)
                filtered[indices] = probs[indices]
                filtered /= filtered.sum()
                probs = filtered
            probs = probs / probs.sum()
            return int(np.random.choice(len(probs), p=probs))
        return int(np.argmax(logits))

    def generate(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                 temperature: float = 1.0, top_k: int = 0,
                 eos_token_id: int | None = None) -> np.ndarray:
        """Autoregressive generation with KV cache (model.py:440-500)."""
        token_ids = np.asarray(token_ids)
        if token_ids.shape[0] != 1:
            raise ValueError(f"Batch size must be 1, got {token_ids.shape[0]}")
        if token_ids.shape[1] == 0:
            raise ValueError("token_ids must have at least 1 token")
        total_tokens = token_ids.shape[1] + max_new_tokens
        if total_tokens > self.config.n_positions:
            raise ValueError(
                f"total tokens ({total_tokens} = {token_ids.shape[1]} prompt "
                f"+ {max_new_tokens} new) exceeds n_positions "
                f"({self.config.n_positions})")
        self._init_cache(total_tokens)
        logits = self.forward(token_ids, use_cache=True)
        tokens = [int(t) for t in token_ids[0]]
        for step in range(max_new_tokens):
            nxt = self._sample(logits[0, -1, :], temperature, top_k)
            tokens.append(nxt)
            if nxt == eos_token_id:
                break
            if step < max_new_tokens - 1:
                logits = self.forward(np.array([[nxt]], dtype=np.int32), use_cache=True)
        return np.array([tokens], dtype=np.int32)

    def generate_gpu(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                     temperature: float = 1.0, top_k: int = 0,
                     eos_token_id: int | None = None) -> np.ndarray:
        """Server-facing alias (model.py:502-517)."""
        return self.generate(token_ids, max_new_tokens=max_new_tokens,
                             temperature=temperature, top_k=top_k,
                             eos_token_id=eos_token_id)

    def generate_stream_gpu(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                            temperature: float = 1.0, top_k: int = 0,
                            eos_token_id: int | None = None):
        """Yields (token_id, step_time_s) (model.py:519-554)."""
        token_ids = np.asarray(token_ids)
        if token_ids.shape[0] != 1:
            raise ValueError(f"Batch size must be 1, got {token_ids.shape[0]}")
        if token_ids.shape[1] == 0:
            raise ValueError("token_ids must have at least 1 token")
        self._init_cache(min(self.config.n_positions, token_ids.shape[1] + max_new_tokens))
        t0 = time.perf_counter()
        logits = self.forward(token_ids, use_cache=True)
        nxt = self._sample(logits[0, -1, :], temperature, top_k)
        yield nxt, time.perf_counter() - t0
        if nxt == eos_token_id:
            return
        for _ in range(max_new_tokens - 1):
            t0 = time.perf_counter()
            logits = self.forward(np.array([[nxt]], dtype=np.int32), use_cache=True)
            nxt = self._sample(logits[0, -1, :], temperature, top_k)
            yield nxt, time.perf_counter() - t0
            if nxt == eos_token_id:
                return
