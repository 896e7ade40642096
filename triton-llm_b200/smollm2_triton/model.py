"""SmolLM2 / Llama inference model (drop-in for smollm2_triton/model.py).

``SmolLM2ForCausalLM`` keeps the reference's constructor and methods
(model.py:24-620): ``_init_cache_gpu`` / ``_init_cache``, ``_forward_cached``,
``forward_gpu`` / ``forward``, ``generate_gpu`` / ``generate``,
``generate_stream_gpu`` / ``generate_stream``, ``_embed``, ``_sample``, the
``kv_cache_dev[layer]["k"]`` tensors of shape (n_kv_head, max_seq, d_k) and
``_cache_len``. Underneath, the batched engine (engine.py) runs every step on
the GPU: the KV cache is written and read in place (the reference copies the
whole prefix between host and device in every layer, model.py:301-308), and
decode steps sample on the device, greedy or temperature / top-k.

``generate_batch`` adds ragged-batch greedy generation over many prompts.
"""

from __future__ import annotations

import time

import numpy as np

from triton_llm import gpu
from .config import SmolLM2Config
from .engine import LlamaSession, LlamaWeights


class SmolLM2ForCausalLM:
    """SmolLM2 (Llama-architecture) model on sm_100a kernels.

    Parameters
    ----------
    config : SmolLM2Config
    weights : dict of str -> np.ndarray
        HuggingFace names and (out_features, in_features) Linear layouts.
    dtype : "float32" | "bfloat16" | None
        Storage precision of weights and KV cache (default:
        ``config.torch_dtype``). Activations and accumulation are fp32.
    kv_dtype : "float32" | "bfloat16" | None
        KV cache precision when it should differ from ``dtype``.
    act_dtype : "split" | "bfloat16"
        Projection inputs of the bf16 path: hi + lo bf16 planes (default:
        ~16 mantissa bits, close to the reference's fp32 activations, twice
        the tensor-core work), or one bf16 plane (faster; its rounding can
        flip a greedy token where the reference's top two logits are within
        ~1e-5).
    """

    @classmethod
    def from_safetensors(cls, path, config: SmolLM2Config | None = None, **kw):
        """Build from a safetensors checkpoint (a file, a list of shards, or a
        directory with ``model.safetensors`` or an index and its shards; the
        directory's ``config.json`` gives the config when none is passed).
        Tensors are read from the memory-mapped files one at a time."""
        import json
        import os
        from triton_llm.safetensors import load_state_dict
        if config is None:
            cj = os.path.join(path, "config.json") if os.path.isdir(str(path)) else None
            if not cj or not os.path.exists(cj):
                raise ValueError("pass a config, or a directory holding config.json")
            with open(cj) as f:
                config = SmolLM2Config.from_dict(json.load(f))
        return cls(config, load_state_dict(path), **kw)

    def __init__(self, config: SmolLM2Config, weights: dict, dtype: str | None = None,
                 kv_dtype: str | None = None, act_dtype: str = "split"):
        self.config = config
        if config.n_head % config.n_kv_head != 0:
            raise ValueError(
                f"n_head ({config.n_head}) must be divisible by n_kv_head ({config.n_kv_head})")
        if "lm_head.weight" not in weights and not config.tie_word_embeddings:
            raise KeyError("lm_head.weight is missing from weights and tie_word_embeddings is False")
        self.wte = np.require(weights["model.embed_tokens.weight"], dtype=np.float32,
                              requirements=["C_CONTIGUOUS"])
        self._weights = weights
        self._dtype = dtype
        self._kv_dtype = kv_dtype
        self._act_dtype = act_dtype
        self._gpu_initialized = False
        self.dev: LlamaWeights | None = None
        self.session: LlamaSession | None = None
        self.kv_cache_dev = None
        self._cache_len = 0

    # ------------------------------------------------------------------
    def _init_gpu_weights(self):
        """Upload the weights once (smollm2_triton/model.py:163-184)."""
        if self._gpu_initialized:
            return
        self.dev = LlamaWeights(self.config, self._weights, self._dtype)
        self._gpu_initialized = True

    def _init_cache_gpu(self, max_seq: int | None = None):
        """Preallocate the KV cache (smollm2_triton/model.py:190-225)."""
        if max_seq is None:
            max_seq = self.config.max_position_embeddings
        elif max_seq <= 0:
            raise ValueError(f"max_seq must be a positive integer, got {max_seq}")
        elif max_seq > self.config.max_position_embeddings:
            raise ValueError(
                f"max_seq ({max_seq}) cannot exceed model's "
                f"max_position_embeddings ({self.config.max_position_embeddings})")
        self._init_gpu_weights()
        if self.session is None or self.session.S != max_seq or self.session.B != 1:
            self.session = LlamaSession(self.dev, 1, max_seq, kv_dtype=self._kv_dtype,
                                        act_dtype=self._act_dtype)
        else:
            gpu.memset(self.session.kv_arena, 0)
        d = self.dev
        self.kv_cache_dev = [
            {"k": gpu.view(k, (d.Hkv, max_seq, d.D)), "v": gpu.view(v, (d.Hkv, max_seq, d.D))}
            for (k, v) in self.session.kv]
        self._cache_len = 0

    # ------------------------------------------------------------------
    def _forward_cached(self, token_ids: np.ndarray) -> np.ndarray:
        """Cached forward pass (smollm2_triton/model.py:231-379).

        Prefill when the cache is empty (any length), otherwise one decode
        token. Returns host logits (1, seq, vocab_size) float32.
        """
        self._init_gpu_weights()
        if self.kv_cache_dev is None:
            raise RuntimeError("_init_cache_gpu() must be called before _forward_cached()")
        token_ids = np.asarray(token_ids)
        prev_seq = self._cache_len
        seq = token_ids.shape[1]
        if prev_seq != 0 and seq > 1:
            raise ValueError(f"Decode mode requires seq=1, got seq={seq}. ")
        total_after = prev_seq + seq
        max_seq = self.session.S
        if total_after > max_seq:
            raise ValueError(f"Total sequence length {total_after} exceeds "
                             f"pre-allocated cache size ({max_seq})")
        s = self.session
        if prev_seq == 0:
            logits = s.prefill([token_ids[0]], all_logits=True)
        else:
            s.set_state(np.array([prev_seq], np.int32),
                        np.array([int(token_ids[0, 0])], np.int32))
            s.decode_step(sample=False)
            logits = s.logits.to_numpy()[:1]
        self._cache_len = total_after
        return logits.reshape(1, seq, self.config.vocab_size)

    def forward_gpu(self, token_ids: np.ndarray, use_cache: bool = False) -> np.ndarray:
        """Forward pass (smollm2_triton/model.py:381-406)."""
        token_ids = np.asarray(token_ids)
        if token_ids.ndim != 2 or token_ids.shape[0] != 1 or token_ids.shape[1] == 0:
            raise ValueError(
                f"token_ids must be a non-empty 2D array with shape (1, seq), "
                f"got shape {token_ids.shape}")
        if use_cache:
            if self.kv_cache_dev is None:
                raise RuntimeError(
                    "_init_cache_gpu() must be called before forward_gpu(use_cache=True)")
        else:
            self._init_cache_gpu(max_seq=min(self.config.max_position_embeddings,
                                             max(token_ids.shape[1], 1)))
        return self._forward_cached(token_ids)

    # ------------------------------------------------------------------
    def _validate(self, token_ids, max_new_tokens, temperature, top_k):
        if token_ids.shape[0] != 1:
            raise ValueError(f"Batch size must be 1, got {token_ids.shape[0]}")
        if token_ids.shape[1] == 0:
            raise ValueError("token_ids must have at least 1 token")
        if temperature < 0.0:
            raise ValueError("temperature must be non-negative")
        if top_k < 0:
            raise ValueError("top_k must be non-negative")
        total_tokens = token_ids.shape[1] + max_new_tokens
        if total_tokens > self.config.max_position_embeddings:
            raise ValueError(
                f"total tokens ({total_tokens} = {token_ids.shape[1]} prompt "
                f"+ {max_new_tokens} new) exceeds max_position_embeddings "
                f"({self.config.max_position_embeddings})")

    def enable_batching(self, max_batch: int = 8, max_seq: int | None = None):
        """Serve greedy generate_gpu / generate_stream_gpu calls from any
        thread through one batched session (``BatchScheduler``): concurrent
        requests share each decode step instead of queueing behind each
        other. Sampling with temperature keeps the single-request path."""
        from .engine import LlamaSession
        from .scheduler import BatchScheduler
        self.disable_batching()
        self._init_gpu_weights()
        S = int(max_seq or self.config.max_position_embeddings)
        self._sched = BatchScheduler(
            lambda B, S: LlamaSession(self.dev, B, S, kv_dtype=self._kv_dtype,
                                      act_dtype=self._act_dtype),
            max_batch, S)
        return self._sched

    def disable_batching(self):
        if getattr(self, "_sched", None) is not None:
            self._sched.close()
            self._sched = None

    def generate_gpu(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                     temperature: float = 1.0, top_k: int = 0,
                     eos_token_id: int | None = None) -> np.ndarray:
        """Autoregressive generation (smollm2_triton/model.py:408-469).

        Returns (1, seq + generated) int32. Every decode step samples on the
        device (argmax when temperature <= 1e-6, else temperature / top-k with
        the uniform drawn from NumPy's global generator, as the reference's
        np.random.choice draws it); the first token, from the prompt's
        logits, is drawn by ``_sample`` on the host like the reference.
        """
        token_ids = np.asarray(token_ids)
        self._validate(token_ids, max_new_tokens, temperature, top_k)
        if getattr(self, "_sched", None) is not None and temperature <= 1e-6:
            out = self._sched.generate(token_ids[0], max_new_tokens, eos_token_id)
            return out.reshape(1, -1).astype(np.int32)
        out = [int(t) for t in token_ids[0]]
        for tok, _ in self._stream(token_ids, max_new_tokens, temperature, top_k,
                                   eos_token_id):
            out.append(tok)
        return np.array([out], dtype=np.int32)

    def generate_stream_gpu(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                            temperature: float = 1.0, top_k: int = 0,
                            eos_token_id: int | None = None):
        """Yields (token_id, step_time_s): TTFT first, then per-token time
        (smollm2_triton/model.py:471-541)."""
        token_ids = np.asarray(token_ids)
        self._validate(token_ids, max_new_tokens, temperature, top_k)
        if getattr(self, "_sched", None) is not None and temperature <= 1e-6:
            yield from self._sched.submit(token_ids[0], max_new_tokens, eos_token_id).stream()
            return
        yield from self._stream(token_ids, max_new_tokens, temperature, top_k,
                                eos_token_id)

    def _stream(self, token_ids, max_new_tokens, temperature, top_k, eos_token_id):
        greedy = temperature <= 1e-6
        total = token_ids.shape[1] + max_new_tokens
        self._init_cache_gpu(max_seq=max(total, 1))
        s = self.session
        t0 = time.perf_counter()
        logits = self._forward_cached(token_ids)
        t_step = t0
        for step in range(max_new_tokens):
            if step == 0:
                tok = self._sample(logits[0, -1, :], temperature, top_k)
            else:
                tok = int(s.ids.to_numpy()[0])
            yield tok, time.perf_counter() - t_step
            if eos_token_id is not None and tok == eos_token_id:
                return
            if step < max_new_tokens - 1:
                t_step = time.perf_counter()
                s.set_state(np.array([self._cache_len], np.int32),
                            np.array([tok], np.int32))
                if not greedy:
                    # the one uniform np.random.choice would draw this step
                    s.u.from_numpy(np.array([np.random.random_sample()], np.float64))
                s.decode_step(sample=True, temperature=temperature, top_k=top_k)
                self._cache_len += 1

    def generate_batch(self, prompts, max_new_tokens: int = 20,
                       eos_token_id: int | None = None, use_graph: bool = True):
        """Greedy generation for several prompts at once (ragged lengths).

        Returns a list of int32 arrays (prompt + generated tokens). Each step
        is one CUDA graph launch; generation stops at max_new_tokens (tokens
        after an eos are dropped from the returned sequence).
        """
        prompts = [np.asarray(p, np.int32).reshape(-1) for p in prompts]
        longest = max(len(p) for p in prompts) + max_new_tokens
        if longest > self.config.max_position_embeddings:
            raise ValueError(f"{longest} tokens exceed max_position_embeddings "
                             f"({self.config.max_position_embeddings})")
        self._init_gpu_weights()
        sess = LlamaSession(self.dev, len(prompts), longest, kv_dtype=self._kv_dtype,
                            act_dtype=self._act_dtype)
        logits = sess.prefill(prompts)
        gen = [[int(np.argmax(logits[b]))] for b in range(len(prompts))]
        if use_graph and max_new_tokens > 1:
            sess.capture()
        for _ in range(max_new_tokens - 1):
            sess.step()
            ids = sess.ids.to_numpy()
            for b in range(len(prompts)):
                gen[b].append(int(ids[b]))
        out = []
        for p, g in zip(prompts, gen):
            if eos_token_id is not None and eos_token_id in g:
                g = g[: g.index(eos_token_id) + 1]
            out.append(np.concatenate([p, np.array(g, np.int32)]))
        return out

    # ------------------------------------------------------------------
    def _embed(self, token_ids: np.ndarray) -> np.ndarray:
        """Host token embedding lookup (smollm2_triton/model.py:547-560)."""
        return self.wte[token_ids.ravel()].reshape(token_ids.shape[0], token_ids.shape[1], -1)

    def _sample(self, logits: np.ndarray, temperature: float, top_k: int) -> int:
        """Greedy or temperature / top-k sampling (model.py:566-584)."""
        if temperature > 1e-6:
            scaled = logits / temperature
            logits_stable = scaled - np.max(scaled)
            probs = np.exp(logits_stable).astype(np.float64)
            probs = probs / np.sum(probs)
            if top_k > 0:
                top_k = min(top_k, len(probs))
                indices = np.argpartition(probs, -top_k)[-top_k:]
                filtered = np.zeros_like(probs)
                filtered[indices] = probs[indices]
                filtered /= filtered.sum()
                probs = filtered
            return int(np.random.choice(len(probs), p=probs))
        return int(np.argmax(logits))

    # ------------------------------------------------------------------
    # Aliases kept by the reference (model.py:590-620)
    def _init_cache(self, max_seq: int | None = None):
        return self._init_cache_gpu(max_seq)

    def forward(self, token_ids: np.ndarray, use_cache: bool = False) -> np.ndarray:
        return self.forward_gpu(token_ids, use_cache)

    def generate(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                 temperature: float = 1.0, top_k: int = 0,
                 eos_token_id: int | None = None) -> np.ndarray:
        return self.generate_gpu(token_ids, max_new_tokens, temperature, top_k,
                                 eos_token_id=eos_token_id)

    def generate_stream(self, token_ids: np.ndarray, max_new_tokens: int = 20,
                        temperature: float = 1.0, top_k: int = 0,
                        eos_token_id: int | None = None):
        yield from self.generate_stream_gpu(token_ids, max_new_tokens, temperature,
                                            top_k, eos_token_id=eos_token_id)
