"""Benchmark of the B200 decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl b200|reference] [--no-cpu-baseline]

Prints ONE JSON line on rank 0. Under torchrun (N > 1) every rank drives
its own GPU (a data-parallel replica, or a tensor-parallel shard for
llama3b_tp); ranks meet at host barriers around the timed regions over the
package's TCP rendezvous (triton_llm.rendezvous, MASTER_PORT + 1), and every
time reported is the maximum over ranks.

Workloads:
  llama3b  (default) config 4: Llama-3.2-3B architecture, bf16 weights and
           KV cache, random-init weights N(0, 0.02); one ragged batch of 64
           sequences whose cached contexts are uniform in [1024, 8192] (K/V
           filled N(0, 1)); K greedy decode steps. The 64 lengths come from
           one seeded stream and are partitioned across the N ranks (64 / N
           each) balancing total context (triton_llm.shard), so the total
           work is fixed as N grows (strong scaling).
  llama3b_weak  the same with 64 sequences on every rank (weak scaling).
  gqa      config 2: the isolated split-KV GQA decode-attention kernel, 64
           ragged sequences (U[128, 2048], seed 1), 9 q / 3 kv heads,
           head_dim 64, bf16 cache; one step = one launch over the batch.

value = decode tokens/s of the whole job (device time of K steps, each step
one CUDA-graph replay of the whole decode step, inputs resident in HBM).
e2e   = the same through the serving loop with host token buffers: every step
copies the batch's token ids from pinned host memory, replays the step and
reads the sampled ids back.
roofline = the dominant kernel (split-KV attention), timed in an
attention-only graph replay of the step's L layer launches on the same cache
right after the timed region, with its algorithmic bytes per launch.

The reference arm (--impl reference) times the reference's math on the host
cores: the CPU oracle (oracle/, a numpy restatement of the reference's
model and kernels) on a bounded sample of the same workload, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

# The reference arm times numpy on every host core; torchrun pins
# OMP_NUM_THREADS=1, so the BLAS thread counts are set before numpy loads.
if "reference" in sys.argv:
    _n = str(len(os.sched_getaffinity(0)))
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = _n

# NCCL prints its version line on stdout at init; the bench's stdout is one
# JSON line (NCCL_DEBUG set explicitly is kept).
os.environ.setdefault("NCCL_DEBUG", "NONE")

import numpy as np  # noqa: E402

REPO = Path(__file__).resolve().parent
for _p in (REPO / "triton-llm_b200", REPO, REPO / "tests" / "golden"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "decode tokens/s (whole box)"
FALLBACK_HBM_GBS = 6650.0


# ------------------------------------------------------------------ ranks ----
class Ranks:
    """This process's rank; ranks meet over the package's TCP rendezvous
    (triton_llm.rendezvous: host barriers and max / sum of host numbers, no
    torch.distributed)."""

    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.rdzv = None
        if self.world > 1:
            from triton_llm.rendezvous import Rendezvous
            self.rdzv = Rendezvous.from_env(timeout=600.0)

    def barrier(self):
        if self.rdzv:
            self.rdzv.barrier()

    def max(self, x: float) -> float:
        return self.rdzv.reduce_max(x) if self.rdzv else x

    def sum(self, x: float) -> float:
        return self.rdzv.reduce_sum(x) if self.rdzv else x

    def close(self):
        if self.rdzv:
            self.rdzv.barrier()
            self.rdzv.close()


# ----------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi sampled every 200 ms during a timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [x for x in (num(r[1]) for r in rows) if x is not None]
        mx = [x for x in (num(r[2]) for r in rows) if x is not None]
        pw = [x for x in (num(r[3]) for r in rows) if x is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(key: str, alg_bytes: int | None = None):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary
    (profiles/traffic.json), or None. When the summary records the ratio of
    DRAM traffic to algorithmic bytes and ``alg_bytes`` is given, the
    traffic of this launch is that ratio times its algorithmic bytes (the
    capture's case and this launch differ only in the contexts read, which
    traffic follows in proportion); else the captured launch's bytes."""
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        try:
            d = json.loads(p.read_text()).get(key)
            if not d:
                return None
            r = d.get("traffic_over_algorithmic")
            if r and alg_bytes:
                return int(round(r * alg_bytes))
            return d.get("bytes_per_launch")
        except Exception:
            return None
    return None


def _time_graph(gpu, graph, reps):
    """Mean ms of one replay of ``graph`` over ``reps`` replays (events on
    the library stream, one untimed replay first)."""
    graph.launch()
    gpu.device_synchronize()
    e0, e1 = gpu.Event(), gpu.Event()
    e0.record()
    for _ in range(reps):
        graph.launch()
    e1.record()
    gpu.device_synchronize()
    return e0.elapsed_ms(e1) / reps


# -------------------------------------------------------- config 4: Llama ----
class LlamaDecodeWorkload:
    """Llama-3.2-3B ragged-batch decode (bf16), one batch
    of 64 sequences split over the N ranks (64 / N each, strong scaling)."""

    name = "llama3b"
    scaling = "strong"
    dtype = "bf16"
    act = "split"
    model = "Llama-3.2-3B-Instruct"
    global_batch = 64        # per_rank = global_batch / N
    per_rank = None          # fixed per-rank batch instead (weak scaling)
    lo, hi = 1024, 8192
    len_seed = 4

    def __init__(self, ranks, steps, warmup):
        from triton_llm import shard
        self.ranks = ranks
        self.steps, self.warmup = steps, warmup
        n = ranks.world
        if self.per_rank is None:
            if self.global_batch % n:
                raise SystemExit(f"{self.global_batch} sequences do not split over {n} GPUs")
            per = self.global_batch // n
        else:
            per = self.per_rank
        self.all_lens = shard.ragged_lengths(per * n, self.lo, self.hi, self.len_seed)
        self.parts = shard.partition(self.all_lens, n, per)
        self.idx = self.parts[ranks.rank]
        self.lens = self.all_lens[self.idx].astype(np.int32)
        self.B = len(self.lens)
        # room for the warm-up and timed steps after the longest context
        self.S = ((self.hi + steps + warmup + 2 + 63) // 64) * 64

    def config(self):
        n = self.ranks.world
        split = ("one batch split over the GPUs" if self.per_rank is None
                 else f"{self.per_rank} sequences per GPU")
        return {"workload": "cfg4 Llama-3.2-3B ragged-batch greedy decode",
                "model": self.model, "layers": 28, "hidden": 3072,
                "heads": "24 q / 8 kv, head_dim 128", "ffn": 8192, "vocab": 128256,
                "batch_per_gpu": self.B, "global_batch": self.B * n,
                "batching": split,
                "ctx": f"U[{self.lo},{self.hi}] seed {self.len_seed}, "
                       "partitioned by total context",
                "sum_ctx_this_rank": int(self.lens.sum()),
                "weights": "random N(0,0.02) bf16 (seed 0), tied embeddings",
                "projection_inputs": ("bf16 hi/lo planes" if self.act == "split" else "bf16"),
                "kv_cache": f"bf16 (B, 8, {self.S}, 128) per layer, filled N(0,1)",
                "parallelism": f"dp{self.ranks.world} (independent replicas, no collective)",
                "timed": "K steps, each one CUDA-graph replay of the full decode step "
                         "(embedding, 28 x [rmsnorm, qkv+rope+append, attention, o+resid, "
                         "rmsnorm, gate/up+swiglu, down+resid], norm, lm_head, argmax)",
                "l2": "inputs larger than L2: every step reads all weights (6.4 GB) and "
                      "the whole cached context (~34 GB) once"}

    def setup(self):
        from triton_llm import gpu, _lib
        from smollm2_triton import SmolLM2Config
        from smollm2_triton.engine import LlamaSession, LlamaWeights
        self.gpu = gpu
        cfg = SmolLM2Config.from_pretrained(self.model)
        self.cfg = cfg
        self.wts = LlamaWeights(cfg, None, "bfloat16", seed=0, std=0.02, max_pos=self.S)
        self.sess = LlamaSession(self.wts, self.B, self.S, act_dtype=self.act)
        s = self.sess
        self.fill_context()
        self.reset()
        self.launches_per_step = s.decode_step(True)
        gpu.device_synchronize()
        self.reset()
        # pinned token buffers of the serving loop
        self.ids_host = gpu.pinned_empty((self.B,), np.int32)
        self.out_host = gpu.pinned_empty((self.B,), np.int32)
        self.h2d = self.B * 4
        self.d2h = self.B * 4

    def fill_context(self):
        """The cached contexts: K/V filled N(0, 1) on the device (a
        counter-based generator) and random next tokens."""
        from triton_llm import _lib
        s = self.sess
        _lib.call("tllm_fill_random", s.kv_arena.ptr, _lib.BF16,
                  int(np.prod(s.kv_arena.shape)), 1000 + self.ranks.rank, 1.0, None)
        rng = np.random.default_rng(100)
        all_ids = rng.integers(0, self.cfg.vocab_size, len(self.all_lens)).astype(np.int32)
        self.ids0 = all_ids[self.idx]

    def reset(self):
        self.sess.set_state(self.lens, self.ids0)

    def capture(self):
        self.sess.capture()

    def step(self):
        self.sess.step()

    def units_per_step(self):
        return self.B

    def e2e_begin(self):
        self.reset()
        self.ids_host[...] = self.ids0

    def step_e2e(self):
        self.sess.step_host(self.ids_host, self.out_host)
        self.ids_host[...] = self.out_host

    # ---- dominant kernel: attention, timed alone on the same cache ----
    def kernel_roofline(self, gpu, peak):
        from triton_llm.kernels import gqa_rows
        s, w = self.sess, self.wts
        g = gpu.Graph()
        with g:
            for i in range(w.L):
                k, v = s.kv[i]
                gqa_rows(s.q, k, v, s.row_seq, s.lens, s.attn, s.B, w.H, w.H * w.D,
                         w.D, w.H * w.D, w.D, s.S, workspace=s.attn_ws,
                         keys_hint=s._keys_hint)   # the step's own split plan
        ms = _time_graph(gpu, g, 5) / w.L
        lens = s.lens.to_numpy().astype(np.int64)
        alg = (2 * w.Hkv * w.D * 2 * int(lens.sum())            # K and V, bf16
               + 2 * s.B * w.H * w.D * 4 + s.B * 4)             # q, out, lens
        achieved = alg / (ms / 1e3) / 1e9
        return {"kernel": "gqa_decode_mma_kernel<128, 1, 1> (+ split merge)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "bound": "hbm",
                "algorithmic_bytes_per_launch": alg,
                "launch_ms": round(ms, 5),
                "timing": f"attention-only CUDA graph of the {w.L} layer launches of "
                          "one step on the same cache, 5 replays, CUDA events",
                "traffic": profiled_traffic("llama3b_attention", alg),
                "traffic_source": "ncu DRAM read+write / algorithmic bytes of one "
                                  "config-4 layer launch (profiles/traffic.json), "
                                  "times this launch's algorithmic bytes"}

    def projection_roofline(self, gpu, peak):
        """All projection GEMMs of one step replayed alone (weights stream)."""
        from triton_llm import _lib
        from triton_llm.kernels.linear import linear
        from triton_llm.kernels.mlp import mlp_block
        s, w = self.sess, self.wts
        B = s.B
        g = gpu.Graph()
        alg = 0
        with g:
            for i in range(w.L):
                L = w.layers[i]
                k, v = s.kv[i]
                linear(s.x, L["qkv"], op=_lib.EPI_QKV, ws=s.lin_ws, M=B, qkv=dict(
                    cos=w.cos, sin=w.sin, row_seq=s.row_seq, row_pos=s.pos, q_out=s.q,
                    k_cache=k, v_cache=v, n_head=w.H, n_kv_head=w.Hkv, head_dim=w.D))
                if s.mlp_ws is not None:
                    # the step's own form: o, norm, gate/up, down in one launch
                    mlp_block(s.attn, L["o"], s.h, L["ln2"], s.x, L["gu"], s.act, L["down"],
                              B, w.eps, s.mlp_ws)
                else:
                    linear(s.attn, L["o"], out_dev=s.x, op=_lib.EPI_STORE, ws=s.lin_ws, M=B)
                    linear(s.x, L["gu"], out_dev=s.act, op=_lib.EPI_SWIGLU, ws=s.lin_ws, M=B)
                    linear(s.act, L["down"], out_dev=s.x, op=_lib.EPI_STORE, ws=s.lin_ws, M=B)
            linear(s.x, w.lm_head, out_dev=s.logits, ws=s.lin_ws, M=B)
        for (M, N, K) in w.linear_shapes(B)[:4]:
            alg += w.L * (N * K * 2 + M * K * 4 + M * N * 4)
        M, N, K = w.linear_shapes(B)[4]
        alg += N * K * 2 + M * K * 4 + M * N * 4
        n_launch = (2 if s.mlp_ws is not None else 4) * w.L + 1
        ms = _time_graph(gpu, g, 5)
        achieved = alg / (ms / 1e3) / 1e9
        return {"kernels": projection_kernels(w.linear_shapes(B), s.mlp_ws is not None),
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "bound": "hbm",
                "algorithmic_bytes_per_step": alg, "ms_per_step": round(ms, 4),
                "launches_per_step": n_launch,
                "timing": "projection-only CUDA graph of one step, 5 replays"}

    def check(self):
        """Last layer's attention of the last step for two sequences vs the
        oracle, on the device's own q and cache."""
        from oracle import ops
        gpu, s, w = self.gpu, self.sess, self.wts
        k, v = s.kv[w.L - 1]
        n = 2
        shp = (n, w.Hkv, s.S, w.D)
        kc = gpu.to_host(gpu.sub_view(k, 0, shp))
        vc = gpu.to_host(gpu.sub_view(v, 0, shp))
        q = s.q.to_numpy()[:n]
        lens = s.lens.to_numpy()[:n]
        out = gpu.split_to_host(s.attn, n).reshape(n, w.H, w.D)
        ref = ops.gqa_decode(q, kc, vc, lens)
        return float(np.abs(out - ref).max())


class LlamaWeakWorkload(LlamaDecodeWorkload):
    """Config 4's model and contexts with 64 sequences on EVERY GPU (the
    per-GPU work fixed as N grows: weak scaling)."""

    name = "llama3b_weak"
    scaling = "weak"
    per_rank = 64


class LlamaTPWorkload(LlamaDecodeWorkload):
    """Llama-3.2-3B long-context decode, 8 sequences at a
    32768-token cached context (K/V N(0, 1)), tensor-parallel by KV head over
    the N ranks (each holds 8/N KV heads, 24/N query heads and 8192/N of the
    FFN; o_proj and down_proj partial sums are all-reduced and added to the
    residual by the next RMSNorm: by default the projection epilogue scatters
    its rows to every rank over NVLink and the RMSNorm sums them,
    TLLM_TP_P2P=0 uses NCCL instead). Every rank serves the same
    sequences, so the total work is fixed as N grows (strong scaling)."""

    name = "llama3b_tp"
    scaling = "strong"
    per_rank = 8
    ctx = 32768

    def __init__(self, ranks, steps, warmup):
        self.ranks = ranks
        self.steps, self.warmup = steps, warmup
        self.B = 8
        self.lens = np.full(self.B, self.ctx, np.int32)
        self.S = ((self.ctx + steps + warmup + 2 + 63) // 64) * 64
        self.graph_note = ""
        self.comm = ""

    def config(self):
        n = self.ranks.world
        return {"workload": "cfg5 Llama-3.2-3B long-context greedy decode, KV-head TP",
                "model": self.model, "layers": 28, "hidden": 3072,
                "heads": "24 q / 8 kv, head_dim 128", "ffn": 8192, "vocab": 128256,
                "batch": self.B, "global_batch": self.B, "ctx": self.ctx,
                "parallelism": f"tp{n} by KV head ({8 // n} kv / {24 // n} q heads, "
                               f"ffn {8192 // n} per rank), all-reduce after "
                               "o_proj and down_proj: " + self.comm + ", replicated "
                               "embedding / lm_head",
                "weights": "random N(0,0.02) bf16 (seed 0)",
                "kv_cache": f"bf16 (8, {8 // n}, {self.S}, 128) per layer per rank, N(0,1)",
                "timed": "K steps, each one CUDA-graph replay of the full decode step "
                         "including the all-reduces" + self.graph_note,
                "l2": "inputs larger than L2"}

    def setup(self):
        from triton_llm import gpu, _lib
        from triton_llm.tp import TPGroup
        from smollm2_triton import SmolLM2Config
        from smollm2_triton.engine import LlamaSession, LlamaWeights
        self.gpu = gpu
        r = self.ranks
        self.tp = TPGroup(r.rank, r.world, r.local, rdzv=r.rdzv)
        cfg = SmolLM2Config.from_pretrained(self.model)
        self.cfg = cfg
        self.wts = LlamaWeights(cfg, None, "bfloat16", seed=0, std=0.02, max_pos=self.S,
                                tp_rank=r.rank, tp_size=r.world)
        self.sess = LlamaSession(self.wts, self.B, self.S, act_dtype=self.act, tp=self.tp)
        s = self.sess
        self.comm = ("fused peer-to-peer (projection epilogue stores to every rank over "
                     "NVLink, next RMSNorm sums)" if s.peer is not None else
                     ("NCCL" if r.world > 1 else "none (1 rank)"))
        _lib.call("tllm_fill_random", s.kv_arena.ptr, _lib.BF16,
                  int(np.prod(s.kv_arena.shape)), 2000 + r.rank, 1.0, None)
        self.ids0 = np.random.default_rng(100).integers(0, cfg.vocab_size, self.B).astype(np.int32)
        self.reset()
        self.launches_per_step = s.decode_step(True)
        gpu.device_synchronize()
        self.reset()
        self.ids_host = gpu.pinned_empty((self.B,), np.int32)
        self.out_host = gpu.pinned_empty((self.B,), np.int32)
        self.h2d = self.B * 4
        self.d2h = self.B * 4

    def capture(self):
        try:
            self.sess.capture()
        except Exception as e:  # NCCL inside a graph needs a capturable stream
            self.sess.graph = None
            self.graph_note = f" (graph capture failed, eager launches: {str(e)[:80]})"

    def projection_roofline(self, gpu, peak):
        return None

    def kernel_roofline(self, gpu, peak):
        r = super().kernel_roofline(gpu, peak)
        r["traffic"] = None   # the committed capture is of the config-4 cache
        r.pop("traffic_source", None)
        return r

    def units_per_step(self):
        # every rank serves the same sequences: count them once per job
        return self.B / self.ranks.world


class SmolDecodeWorkload(LlamaDecodeWorkload):
    """SmolLM2-135M, 32 sequences per GPU (bf16): every
    sequence's 512-token prompt (uniform ids, seed 3) runs through the
    model's own prefill (timed apart and reported as ``prefill``), then K
    greedy decode steps continue from position 512 (the configuration's 256
    steps: --steps 256)."""

    name = "smol135m"
    scaling = "weak"
    model = "SmolLM2-135M"
    per_rank = 32
    lo, hi = 512, 512
    prompt_seed = 3

    def fill_context(self):
        from triton_llm import gpu
        s = self.sess
        rng = np.random.default_rng(self.prompt_seed + self.ranks.rank)
        prompts = rng.integers(0, self.cfg.vocab_size, (self.B, self.lo)).astype(np.int32)
        s.prefill(prompts)                      # warm: buffers, kernels
        gpu.device_synchronize()
        e0, e1 = gpu.Event(), gpu.Event()
        t = time.perf_counter()
        e0.record()
        s.prefill(prompts)
        e1.record()
        gpu.device_synchronize()
        wall = time.perf_counter() - t
        ms = e0.elapsed_ms(e1)
        toks = self.B * self.lo
        self.prefill_info = {
            "tokens": toks, "device_ms": round(ms, 3), "wall_ms": round(wall * 1e3, 3),
            "tokens_per_s": round(toks / (ms / 1e3), 1),
            "what": f"{self.B} prompts x {self.lo} tokens through the model's prefill "
                    "(embedding, 30 layers with the causal prefill attention kernel, "
                    "final norm, lm_head of the last rows), host argmax; not part of "
                    "the decode tokens/s"}
        self.ids0 = s.ids.to_numpy().astype(np.int32)

    def config(self):
        w = self.ranks.world
        c = {"workload": "cfg3 SmolLM2-135M batched greedy decode",
             "model": self.model, "layers": 30, "hidden": 576,
             "heads": "9 q / 3 kv, head_dim 64", "ffn": 1536, "vocab": 49152,
             "batch_per_gpu": self.B, "global_batch": self.B * w,
             "prompt": f"{self.lo} uniform ids per sequence (seed {self.prompt_seed}), "
                       "prefilled through the model",
             "ctx": f"{self.lo} .. {self.lo} + K during the timed steps",
             "weights": "random N(0,0.02) bf16 (seed 0), tied embeddings",
             "projection_inputs": ("bf16 hi/lo planes" if self.act == "split" else "bf16"),
             "kv_cache": f"bf16 (B, 3, {self.S}, 64) per layer",
             "parallelism": f"dp{w} (independent replicas, no collective)",
             "timed": "K steps, each one CUDA-graph replay of the full decode step "
                      "(embedding, 30 layers, norm, lm_head, argmax)",
             "l2": "inputs smaller than L2 (269 MB weights + ~0.4 GB KV per step "
                   "exceed it together; no flush)"}
        if getattr(self, "prefill_info", None):
            c["prefill"] = self.prefill_info
        return c

    def kernel_roofline(self, gpu, peak):
        r = super().kernel_roofline(gpu, peak)
        r["kernel"] = "gqa_decode_mma_kernel<64, 1, 2> (+ split merge)"
        r["traffic"] = None
        r.pop("traffic_source", None)
        return r


class GPT2Workload:
    """GPT-2 small (12 x 768, 12 heads, GELU, LayerNorm,
    vocab 50257), fp32 weights N(0, 0.02) from seed 0 in HF order, batch 1:
    a 32-token prompt (uniform ids, seed 0) prefilled, then greedy decode
    steps through the model's own cached forward (``GPT2Model._forward_cached``
    + argmax), the reference's generate loop. Each step brings the (1, V)
    logits to the host like the reference API does."""

    name = "gpt2"
    scaling = "weak"
    dtype = "f32"
    model = "gpt2"

    def __init__(self, ranks, steps, warmup):
        self.ranks = ranks
        self.steps, self.warmup = steps, warmup
        self.prompt_len = 32
        # every phase (2 warm-ups, timed, e2e warm-up, e2e, check) restarts
        # at the prompt; the cache holds the longest of them
        self.S = self.prompt_len + max(steps, warmup) + 8

    def config(self):
        return {"workload": "cfg1 GPT-2 small fp32 greedy decode, batch 1",
                "model": "GPT-2 small (124M)", "layers": 12, "hidden": 768,
                "heads": 12, "ffn": 3072, "vocab": 50257, "batch": 1,
                "prompt": "32 uniform ids (seed 0), prefilled before timing",
                "weights": "N(0,0.02) fp32, seed 0, HF state-dict order",
                "timed": "K decode steps: cached forward of one token (ids, position and "
                         "length to the device, one CUDA-graph replay of its 87 kernels), "
                         "logits to the host, argmax on the host",
                "l2": "inputs larger than L2: 495 MB of fp32 weights per step"}

    def setup(self):
        import inputs
        from triton_llm import gpu
        from gpt2_triton import GPT2Config, GPT2Model
        self.gpu = gpu
        self.cfg = GPT2Config()
        self.w = inputs.gpt2_weights(inputs.GPT2_SMALL, 0)
        self.m = GPT2Model(self.cfg, self.w, dtype="float32")
        self.prompt = np.random.default_rng(0).integers(0, 50257, self.prompt_len).astype(np.int32)
        self.m._init_cache(self.S)
        self.prefill_logits = self.m.forward(self.prompt[None], use_cache=True)[0]
        self.first = int(np.argmax(self.prefill_logits[-1]))
        self.launches_per_step = 87
        self.h2d = 3 * 4 * max(self.m._rows, 1)
        self.d2h = 50257 * 4
        self.reset()

    def reset(self):
        self.m._cache_len = self.prompt_len
        self.tok = self.first

    def capture(self):
        pass   # the model captures its own decode-step graph on first use

    def step(self):
        logits = self.m._forward_cached(np.array([[self.tok]], np.int32))
        self.tok = int(np.argmax(logits[0, -1]))

    def units_per_step(self):
        return 1

    def e2e_begin(self):
        self.reset()

    def step_e2e(self):
        self.step()

    def kernel_roofline(self, gpu, peak):
        """The step's fp32 projections (CUDA-core GEMV) replayed alone."""
        from triton_llm import _lib
        from triton_llm.kernels.linear import linear
        m = self.m
        g = gpu.Graph()
        alg = 0
        with g:
            for L in m.layers:
                for name, op in (("proj", _lib.EPI_STORE), ("fc", _lib.EPI_GELU),
                                 ("mproj", _lib.EPI_STORE)):
                    lin = L[name]
                    src = m.act if name == "mproj" else m.x
                    dst = m.act if name == "fc" else m.h
                    linear(src, lin, out_dev=dst, op=op, ws=m.lin_ws, M=1)
                linear(m.x, L["qkv"], out_dev=m.act, ws=m.lin_ws, M=1)   # 3n <= 4n wide
            linear(m.x, m.lm_head, out_dev=m.logits, ws=m.lin_ws, M=1)
        for L in m.layers:
            for name in ("qkv", "proj", "fc", "mproj"):
                alg += L[name].N * L[name].K * 4
        alg += m.lm_head.N * m.lm_head.K * 4
        ms = _time_graph(gpu, g, 10)
        achieved = alg / (ms / 1e3) / 1e9
        return {"kernel": "linear_f32_kernel (fp32 weights, CUDA cores; 49 launches)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "bound": "hbm",
                "algorithmic_bytes_per_launch": alg, "launch_ms": round(ms, 5),
                "timing": "projection-only CUDA graph of one decode step, 10 replays",
                "traffic": None}

    def projection_roofline(self, gpu, peak):
        return None

    def check(self):
        """Prefill logits of the prompt vs the oracle (fp32 reference math)."""
        from oracle.models import GPT2Oracle
        o = GPT2Oracle(self.cfg, self.w)
        o.init_cache(self.prompt_len + 1)
        want = o.forward_cached(self.prompt[None])[0]
        return float(np.abs(self.prefill_logits - want).max())


def gpt2_cpu_sample(steps: int):
    """The oracle's GPT-2 decode step (numpy, BLAS threads = host cores)
    after the 32-token prompt, median over ``steps``. Returns (tokens/s,
    text)."""
    import inputs
    from oracle.models import GPT2Oracle
    from gpt2_triton import GPT2Config
    cfg = GPT2Config()
    o = GPT2Oracle(cfg, inputs.gpt2_weights(inputs.GPT2_SMALL, 0))
    prompt = np.random.default_rng(0).integers(0, 50257, 32).astype(np.int32)
    o.init_cache(32 + steps + 2)
    logits = o.forward_cached(prompt[None])
    tok = int(np.argmax(logits[0, -1]))
    ts = []
    for _ in range(steps):
        t = time.perf_counter()
        logits = o.forward_cached(np.array([[tok]], np.int32))
        tok = int(np.argmax(logits[0, -1]))
        ts.append(time.perf_counter() - t)
    per = statistics.median(ts)
    return 1.0 / per, (f"oracle GPT-2 small decode step after a 32-token prompt, "
                       f"median of {steps} steps ({per * 1e3:.1f} ms), numpy restatement "
                       "(oracle/), batch 1 like the reference")


def projection_kernels(shapes, fused_mlp: bool) -> str:
    """Which kernel runs each projection of a step (qkv, o, gate/up, down,
    lm_head shapes), grouped by kernel, for the roofline line."""
    from triton_llm.kernels.linear import kernel_name
    names = ["qkv+rope+append", "o", "gate/up+swiglu", "down", "lm_head"]
    groups = {}
    for (M, N, K), nm in zip(shapes, names):
        if fused_mlp and nm in ("o", "gate/up+swiglu", "down"):
            continue
        groups.setdefault(kernel_name(M, N, K), []).append(nm)
    text = " + ".join(f"{k} ({', '.join(v)})" for k, v in groups.items())
    if fused_mlp:
        text += " + mlp_kernel (o, norm, gate/up+swiglu, down in one launch)"
    return text


def llama_cpu_sample(ctx: int, steps: int, model="Llama-3.2-3B-Instruct", log=None):
    """The oracle's decode step for ONE sequence at context ``ctx`` through
    2 of the model's layers and the lm_head, timed with numpy using every
    host core, extrapolated to the full depth. Returns (tokens/s, text)."""
    import dataclasses
    import inputs
    from oracle.models import SmolLM2Oracle
    from smollm2_triton import SmolLM2Config
    full = SmolLM2Config.from_pretrained(model)
    shape = (inputs.LLAMA3B_2L if model.startswith("Llama")
             else dataclasses.replace(inputs.SMOL_135M, num_hidden_layers=2))
    w = inputs.llama_weights(shape, 0)
    cfg = SmolLM2Config(**shape.config_kwargs())
    cfg.max_position_embeddings = ctx + steps + 8
    o = SmolLM2Oracle(cfg, w, weight_dtype="bfloat16")
    del w
    rng = np.random.default_rng(7)
    o.init_cache(ctx + steps + 8)
    for c in o.cache:
        c["k"][:, :ctx] = inputs.bf16_round(rng.standard_normal(c["k"][:, :ctx].shape, dtype=np.float32))
        c["v"][:, :ctx] = inputs.bf16_round(rng.standard_normal(c["v"][:, :ctx].shape, dtype=np.float32))

    from oracle import ops
    n = max(steps, 5)

    def med(fn):
        fn()                                              # warm
        ts = []
        for i in range(n):
            t = time.perf_counter()
            fn(i)
            ts.append(time.perf_counter() - t)
        return statistics.median(ts)

    def step(i=0):
        o.cache_len = ctx
        o.forward_cached(np.array([[i % 1000]], np.int32))

    x = rng.standard_normal((1, cfg.hidden_size), dtype=np.float32)

    def head(i=0):
        ops.gemm(ops.rms_norm(x, o.ln_f, o.eps), o.lm_head_w)

    # the lm_head (final norm + GEMV over the vocabulary) timed alone, then
    # whole 2-layer steps; a layer is the step minus the head, halved
    t_head = med(head)
    t_step = med(step)
    t_layer = max(t_step - t_head, 1e-6) / len(o.layers)
    per_token = t_head + full.num_hidden_layers * t_layer
    text = (f"oracle decode step, 1 sequence at ctx {ctx}: lm_head timed alone "
            f"({t_head * 1e3:.1f} ms) and {len(o.layers)}-layer steps "
            f"({t_step * 1e3:.1f} ms), medians of {n}; per layer {t_layer * 1e3:.1f} ms, "
            f"extrapolated to {full.num_hidden_layers} layers; batch 1 like the "
            "reference, numpy restatement (oracle/)")
    return 1.0 / per_token, text


# ------------------------------------------------- config 2: attention only ----
class GQAWorkload:
    """BASELINE config 2 (isolated GQA decode attention)."""

    name = "gqa"
    scaling = "weak"
    dtype = "bf16"

    COPIES = 6

    def __init__(self, ranks=None, steps=0, warmup=0, copies=COPIES):
        import inputs
        self.ranks = ranks
        self.B, self.H, self.Hkv, self.D, self.S = 64, 9, 3, 64, 2048
        self.lens, self.q, ks, vs = inputs.cfg2_inputs()
        self.kc = inputs.pack_cache(ks, self.S)
        self.vc = inputs.pack_cache(vs, self.S)
        self.copies = copies
        L = int(self.lens.sum())
        self.kv_bytes = 2 * self.Hkv * L * self.D * 2
        self.bytes_per_step = self.kv_bytes + 2 * self.B * self.H * self.D * 4 + self.B * 4
        self.i = 0
        self.graphs = None

    def config(self):
        return {"workload": "cfg2 isolated GQA decode attention",
                "batch": self.B, "n_head": self.H, "n_kv_head": self.Hkv,
                "head_dim": self.D, "kv_lens": "U[128,2048] seed 1",
                "sum_kv_len": int(self.lens.sum()),
                "kv_dtype": "bf16", "kv_layout": "(B, n_kv, 2048, d) prealloc",
                "parallelism": f"dp{self.ranks.world if self.ranks else 1}",
                "timed": "K launches replayed as one CUDA graph",
                "l2": f"{self.COPIES} rotating cache copies "
                      f"({self.COPIES * self.kv_bytes / 1e6:.0f} MB touched > 126 MB L2)"}

    def setup(self):
        from triton_llm import gpu
        from triton_llm.kernels import DecodeWorkspace
        self.gpu = gpu
        kb = gpu.f32_to_bf16_bits(self.kc)
        vb = gpu.f32_to_bf16_bits(self.vc)
        self.kd, self.vd = [], []
        for _ in range(self.copies):
            k = gpu.allocate(kb.shape, gpu.BFLOAT16)
            k.from_numpy(kb)
            v = gpu.allocate(vb.shape, gpu.BFLOAT16)
            v.from_numpy(vb)
            self.kd.append(k)
            self.vd.append(v)
        self.qd = gpu.to_device(self.q)
        self.ld = gpu.to_device(self.lens)
        self.od = gpu.allocate(self.q.shape, np.float32)
        self.ws = DecodeWorkspace(self.B, self.H, self.Hkv, self.D, self.S)
        self.q_host = gpu.pinned_empty(self.q.shape, np.float32)
        self.q_host[...] = self.q
        self.l_host = gpu.pinned_empty(self.lens.shape, np.int32)
        self.l_host[...] = self.lens
        self.o_host = gpu.pinned_empty(self.q.shape, np.float32)
        self.h2d = self.q.nbytes + self.lens.nbytes
        self.d2h = self.q.nbytes
        self.launches_per_step = 1

    def _launch(self):
        from triton_llm.kernels import gqa_decode
        c = self.i % self.copies
        self.i += 1
        gqa_decode(self.qd, self.kd[c], self.vd[c], self.ld, self.od,
                   max_len=self.S, workspace=self.ws)

    def reset(self):
        self.i = 0

    def capture(self):
        # one graph per cache copy; a step replays one launch
        self.i = 0
        graphs = []
        for _ in range(self.copies):
            g = self.gpu.Graph()
            with g:
                self._launch()
            graphs.append(g)
        self.graphs = graphs
        self.i = 0

    def step(self):
        if self.graphs is None:
            self._launch()
            return
        self.graphs[self.i % self.copies].launch()
        self.i += 1

    def units_per_step(self):
        return self.B

    def e2e_begin(self):
        self.i = 0

    def step_e2e(self):
        g = self.gpu
        g.copy_h2d_async(self.qd, self.q_host)
        g.copy_h2d_async(self.ld, self.l_host)
        self.step()
        g.copy_d2h_async(self.o_host, self.od)
        g.stream_synchronize()

    def kernel_roofline(self, gpu, peak):
        ms = None
        e0, e1 = gpu.Event(), gpu.Event()
        reps = 30
        for g in self.graphs:
            g.launch()
        gpu.device_synchronize()
        e0.record()
        for r in range(reps):
            self.graphs[r % self.copies].launch()
        e1.record()
        gpu.device_synchronize()
        ms = e0.elapsed_ms(e1) / reps
        achieved = self.bytes_per_step / (ms / 1e3) / 1e9
        return {"kernel": "gqa_decode_mma_kernel<64, 1, 2> (+ split merge)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "bound": "hbm",
                "algorithmic_bytes_per_launch": self.bytes_per_step,
                "launch_ms": round(ms, 5),
                "timing": f"{reps} graph replays over {self.copies} rotating caches",
                "traffic": profiled_traffic("gqa")}

    def projection_roofline(self, gpu, peak):
        return None

    def check(self):
        from oracle import ops
        out = self.od.to_numpy()
        n = 4
        ref = ops.gqa_decode(self.q[:n], self.kc[:n], self.vc[:n], self.lens[:n])
        return float(np.abs(out[:n] - ref).max())

    # CPU baseline: the oracle on a sample of sequences
    def cpu_run(self, idx):
        from oracle import ops
        ops.gqa_decode(self.q[idx], self.kc[idx], self.vc[idx], self.lens[idx])
        return len(idx)


class _IsolatedWorkload:
    """An isolated kernel at config-4 geometry on device-filled inputs,
    rotating over ``copies`` input sets so the working set exceeds L2.
    A step replays one copy's captured launches."""

    scaling = "weak"
    dtype = "bf16"
    copies = 2

    def __init__(self, ranks=None, steps=0, warmup=0):
        self.ranks = ranks
        self.i = 0
        self.graphs = None

    def reset(self):
        self.i = 0

    def capture(self):
        graphs = []
        for c in range(self.copies):
            g = self.gpu.Graph()
            with g:
                self.launch(c)
            graphs.append(g)
        self.graphs = graphs

    def step(self):
        c = self.i % self.copies
        if self.graphs is None:
            self.launch(c)
        else:
            self.graphs[c].launch()
        self.i += 1

    def e2e_begin(self):
        self.i = 0

    def kernel_roofline(self, gpu, peak):
        reps = 20
        for g in self.graphs:
            g.launch()
        gpu.device_synchronize()
        e0, e1 = gpu.Event(), gpu.Event()
        e0.record()
        for r in range(reps):
            self.graphs[r % self.copies].launch()
        e1.record()
        gpu.device_synchronize()
        ms = e0.elapsed_ms(e1) / reps / self.launches_per_step
        achieved = self.bytes_per_launch / (ms / 1e3) / 1e9
        return {"kernel": self.kernel, "achieved": round(achieved, 1), "peak": peak,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "bound": "hbm",
                "algorithmic_bytes_per_launch": self.bytes_per_launch,
                "launch_ms": round(ms, 5),
                "timing": f"{reps} graph replays over {self.copies} input copies",
                "traffic": profiled_traffic(self.name)}

    def projection_roofline(self, gpu, peak):
        return None


class GQALlamaLayerWorkload(_IsolatedWorkload):
    """Split-KV decode attention alone at config-4 geometry: one layer of
    64 sequences, contexts U[1024, 8192] (seed 4), 24 q / 8 kv heads,
    head_dim 128, bf16 cache filled N(0, 1)."""

    name = "gqa_llama3b"
    kernel = "gqa_decode_mma_kernel<128, 1, 1> (+ split merge)"
    copies = 1      # one launch reads ~1.2 GB, far above L2

    def setup(self):
        from triton_llm import gpu, _lib, shard
        from triton_llm.kernels import DecodeWorkspace
        self.gpu = gpu
        self.B, self.H, self.Hkv, self.D, self.S = 64, 24, 8, 128, 8192
        self.lens = shard.ragged_lengths(self.B, 1024, 8192, 4)
        self.kd, self.vd = [], []
        n = self.B * self.Hkv * self.S * self.D
        for c in range(self.copies):
            for lst, sd in ((self.kd, 2 * c), (self.vd, 2 * c + 1)):
                t = gpu.allocate((self.B, self.Hkv, self.S, self.D), gpu.BFLOAT16)
                _lib.call("tllm_fill_random", t.ptr, _lib.BF16, n, 500 + sd, 1.0, None)
                lst.append(t)
        q = np.random.default_rng(3).standard_normal((self.B, self.H, self.D), dtype=np.float32)
        self.q = q
        self.qd = gpu.to_device(q)
        self.ld = gpu.to_device(self.lens)
        self.od = gpu.allocate(q.shape, np.float32)
        self.ws = DecodeWorkspace(self.B, self.H, self.Hkv, self.D, self.S)
        self.bytes_per_launch = (2 * self.Hkv * self.D * 2 * int(self.lens.sum())
                                 + 2 * q.nbytes + self.lens.nbytes)
        self.launches_per_step = 1
        self.q_host = gpu.pinned_empty(q.shape, np.float32)
        self.q_host[...] = q
        self.o_host = gpu.pinned_empty(q.shape, np.float32)
        self.h2d, self.d2h = q.nbytes, q.nbytes

    def launch(self, c):
        from triton_llm.kernels import gqa_decode
        gqa_decode(self.qd, self.kd[c], self.vd[c], self.ld, self.od,
                   max_len=self.S, workspace=self.ws)

    def units_per_step(self):
        return self.B

    def step_e2e(self):
        g = self.gpu
        g.copy_h2d_async(self.qd, self.q_host)
        self.step()
        g.copy_d2h_async(self.o_host, self.od)
        g.stream_synchronize()

    def config(self):
        return {"workload": "isolated GQA decode attention at cfg4 geometry (one layer)",
                "batch": self.B, "n_head": self.H, "n_kv_head": self.Hkv,
                "head_dim": self.D, "ctx": "U[1024,8192] seed 4",
                "sum_ctx": int(self.lens.sum()), "kv_dtype": "bf16",
                "timed": "K graph replays of one launch",
                "l2": f"{self.copies} rotating caches of "
                      f"{self.bytes_per_launch / 1e9:.2f} GB read per launch"}

    def check(self):
        from oracle import ops
        gpu = self.gpu
        self.launch(0)
        gpu.device_synchronize()
        n = 2
        shp = (n, self.Hkv, self.S, self.D)
        kc = gpu.to_host(gpu.sub_view(self.kd[0], 0, shp))
        vc = gpu.to_host(gpu.sub_view(self.vd[0], 0, shp))
        ref = ops.gqa_decode(self.q[:n], kc, vc, self.lens[:n])
        return float(np.abs(self.od.to_numpy()[:n] - ref).max())


class ProjLlamaLayerWorkload(_IsolatedWorkload):
    """The projection GEMMs of one config-4 decode layer at M = 64 rows:
    qkv (5120 x 3072, RoPE + KV append epilogue), o (3072 x 3072, residual),
    gate/up (16384 x 3072, SwiGLU), down (3072 x 8192, residual); bf16
    weights N(0, 0.02), fp32 activations."""

    name = "proj_llama3b"
    kernel = "linear_tc_kernel<64, op, planes>"
    copies = 4
    planes = 1

    def setup(self):
        from triton_llm import gpu, _lib
        from triton_llm.kernels.linear import Linear, LinearWorkspace
        from triton_llm.kernels.rope import precompute_cos_sin
        self.gpu = gpu
        B, n, H, Hkv, D, F = 64, 3072, 24, 8, 128, 8192
        self.B = B
        self.shapes = [(B, (H + 2 * Hkv) * D, n), (B, n, H * D), (B, 2 * F, n), (B, n, F)]

        def lin(N, K, seed):
            o = Linear.empty_bf16(N, K)
            _lib.call("tllm_fill_random", o.w.ptr, _lib.BF16, int(o.w.shape[0]), seed,
                      0.02, None)
            return o
        self.layers = [[lin(N, K, 10 * c + j) for j, (_, N, K) in enumerate(self.shapes)]
                       for c in range(self.copies)]
        # projection inputs in the tensor-core operand format
        pl = self.planes
        self.x, self.attn, self.act = (gpu.act_empty(B, n, pl), gpu.act_empty(B, H * D, pl),
                                       gpu.act_empty(B, F, pl))
        self.h = gpu.allocate((B, n), np.float32)
        _lib.call("tllm_fill_random", self.h.ptr, _lib.F32, B * n, 2, 1.0, None)
        for t, sd in ((self.x, 1), (self.attn, 3), (self.act, 4)):
            src = gpu.allocate((t.shape[1], t.shape[2]), np.float32)
            _lib.call("tllm_fill_random", src.ptr, _lib.F32, int(np.prod(src.shape)), sd,
                      1.0, None)
            _lib.call("tllm_split_bf16", src.ptr, t.ptr, gpu.act_args(t)[1], t.shape[1],
                      t.shape[2], t.shape[1], None)
        self.q = gpu.allocate((B, H, D), np.float32)
        self.kc = gpu.zeros((B, Hkv, 64, D), gpu.BFLOAT16)
        self.vc = gpu.zeros((B, Hkv, 64, D), gpu.BFLOAT16)
        cos, sin = precompute_cos_sin(64, D, 500000.0)
        self.cos, self.sin = gpu.to_device(cos), gpu.to_device(sin)
        self.row_seq = gpu.to_device(np.arange(B, dtype=np.int32))
        self.pos = gpu.to_device(np.full(B, 7, np.int32))
        self.H, self.Hkv, self.D = H, Hkv, D
        self.ws = LinearWorkspace(self.shapes)
        self.bytes_per_launch = sum(N * K * 2 + M * K * 4 + M * N * 4
                                    for (M, N, K) in self.shapes) // 4
        self.launches_per_step = 4
        self.x_host = gpu.pinned_empty(self.x.shape, np.uint16)
        self.x_host[...] = self.x.to_numpy()
        self.h_host = gpu.pinned_empty((B, n), np.float32)
        self.h2d, self.d2h = self.x.nbytes, B * n * 4

    def launch(self, c):
        from triton_llm import _lib
        from triton_llm.kernels.linear import linear
        qkv, o, gu, down = self.layers[c]
        B = self.B
        linear(self.x, qkv, op=_lib.EPI_QKV, ws=self.ws, M=B, qkv=dict(
            cos=self.cos, sin=self.sin, row_seq=self.row_seq, row_pos=self.pos,
            q_out=self.q, k_cache=self.kc, v_cache=self.vc, n_head=self.H,
            n_kv_head=self.Hkv, head_dim=self.D))
        linear(self.attn, o, out_dev=self.h, op=_lib.EPI_RESID, resid_dev=self.h,
               ws=self.ws, M=B)
        linear(self.x, gu, out_dev=self.act, op=_lib.EPI_SWIGLU, ws=self.ws, M=B)
        linear(self.act, down, out_dev=self.h, op=_lib.EPI_RESID, resid_dev=self.h,
               ws=self.ws, M=B)

    def units_per_step(self):
        return self.B

    def step_e2e(self):
        g = self.gpu
        g.copy_h2d_async(self.x, self.x_host)
        self.step()
        g.copy_d2h_async(self.h_host, self.h)
        g.stream_synchronize()

    def config(self):
        from triton_llm.kernels.linear import plan
        return {"workload": "isolated projection GEMMs of one cfg4 decode layer",
                "rows": self.B, "shapes_MNK": self.shapes,
                "plans": [plan(*sh, planes=self.planes) for sh in self.shapes],
                "weights": "bf16 N(0,0.02)",
                "activations": ("bf16 hi/lo planes (TLLM_SPLIT)" if self.planes == 2
                                else "bf16 (TLLM_BF16)"),
                "timed": "K graph replays of the 4 launches",
                "l2": f"{self.copies} rotating weight sets of 201 MB"}

    def check(self):
        """The gate/up + SwiGLU projection of copy 0 vs numpy in fp64."""
        from oracle import ops
        gpu = self.gpu
        self.launch(0)
        gpu.device_synchronize()
        gu = self.layers[0][2]
        w = gu.to_numpy()[:64].astype(np.float64)         # first 4 blocks of 16 rows
        x = gpu.split_to_host(self.x).astype(np.float64)
        y = x @ w.T                                        # (B, 64) interleaved
        g = np.concatenate([y[:, 16 * b:16 * b + 8] for b in range(4)], axis=1)
        u = np.concatenate([y[:, 16 * b + 8:16 * b + 16] for b in range(4)], axis=1)
        ref = ops.swiglu(g.astype(np.float32), u.astype(np.float32))
        return float(np.abs(gpu.split_to_host(self.act)[:, :32] - ref).max())


WORKLOADS = {"llama3b": LlamaDecodeWorkload, "llama3b_weak": LlamaWeakWorkload,
             "llama3b_tp": LlamaTPWorkload,
             "smol135m": SmolDecodeWorkload, "gpt2": GPT2Workload,
             "gqa": GQAWorkload,
             "gqa_llama3b": GQALlamaLayerWorkload, "proj_llama3b": ProjLlamaLayerWorkload}

# ----------------------------------------------------------- CPU baseline ----
_worker_wl: dict = {}


def _gqa_worker(idx):
    if "gqa" not in _worker_wl:
        _worker_wl["gqa"] = GQAWorkload(copies=0)
    wl = _worker_wl["gqa"]
    t = time.perf_counter()
    n = wl.cpu_run(np.asarray(idx, dtype=np.int64))
    return n, time.perf_counter() - t


def gqa_cpu_baseline(cores, pool, budget_s=15.0):
    """The oracle's attention on a bounded sample of the 64 sequences spread
    over ``cores`` spawned worker processes."""
    warm = pool.map(_gqa_worker, [[0]] * cores)
    per = max(min(r[1] for r in warm), 1e-4)
    nseq = min(max(1, int(budget_s / per)) * cores, 8 * 64)
    idx = np.arange(nseq) % 64
    chunks = [idx[i::cores].tolist() for i in range(cores)]
    t = time.perf_counter()
    res = pool.map(_gqa_worker, [c for c in chunks if c])
    dt = time.perf_counter() - t
    done = sum(r[0] for r in res)
    return done / dt, (f"oracle attention on {done} sequences over {cores} processes "
                       f"({dt:.1f} s); numpy restatement of the reference kernel (oracle/)")


def cpu_baseline(name, cores, steps, pool=None, ctx=None):
    if name == "gqa":
        return gqa_cpu_baseline(cores, pool)
    if name in ("llama3b", "llama3b_weak", "llama3b_tp"):
        return llama_cpu_sample(int(ctx), steps)
    if name == "smol135m":
        return llama_cpu_sample(int(ctx), steps, model=SmolDecodeWorkload.model)
    if name == "gpt2":
        return gpt2_cpu_sample(max(steps, 3))
    return None


# ------------------------------------------------------------------ main ----
def run_b200(args, ranks):
    from triton_llm import gpu
    gpu.set_device(ranks.local)
    gpu.device_error(reset=True)
    wl = WORKLOADS[args.workload](ranks, args.steps, args.warmup)
    wl.setup()
    gpu.device_synchronize()

    # warm-up (eager), then capture the step as a CUDA graph
    wl.reset()
    for _ in range(args.warmup):
        wl.step()
    gpu.device_synchronize()
    wl.capture()
    wl.reset()
    for _ in range(args.warmup):
        wl.step()
    gpu.device_synchronize()
    wl.reset()
    gpu.device_synchronize()

    # timed region: K graph replays between device events, clocks sampled
    clocks = ClockSampler(ranks.local)
    clocks.start()
    ranks.barrier()
    gpu.device_synchronize()
    e0, e1 = gpu.Event(), gpu.Event()
    e0.record()
    for _ in range(args.steps):
        wl.step()
    e1.record()
    gpu.device_synchronize()
    ranks.barrier()
    ms = e0.elapsed_ms(e1)
    clk = clocks.stop()
    ms_max = ranks.max(ms)

    # end-to-end: host token buffers, copies inside the timed region
    wl.e2e_begin()
    for _ in range(2):
        wl.step_e2e()
    wl.e2e_begin()
    ranks.barrier()
    gpu.device_synchronize()
    t0, t1 = gpu.Event(), gpu.Event()
    t0.record()
    for _ in range(args.steps):
        wl.step_e2e()
    t1.record()
    gpu.device_synchronize()
    ranks.barrier()
    e2e_ms = ranks.max(t0.elapsed_ms(t1))

    peak, peak_kind = measured_peaks()
    roof = wl.kernel_roofline(gpu, peak)
    proj = wl.projection_roofline(gpu, peak)
    roof["peak_source"] = ("MEASURED_PEAKS.json hbm_gbs (of measured)"
                           if peak_kind == "measured" else "fallback 6.65 TB/s (of fallback)")
    # one more eager step so the check reads a consistent step
    wl.reset()
    wl.step()
    gpu.device_synchronize()
    err = wl.check()
    dev_err = gpu.device_error()

    units = ranks.sum(wl.units_per_step() * args.steps)
    value = units / (ms_max / 1e3)
    e2e_value = units / (e2e_ms / 1e3)
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": ranks.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 5),
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
        "dtype": wl.dtype, "data": "synthetic (seeded random weights, token ids and "
                                   "KV contents; BASELINE config shapes)",
        "config": wl.config(),
        "roofline": roof,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk,
        "check": {"attention_max_abs_err_vs_oracle": err, "device_error": dev_err},
    }
    if proj:
        out["roofline_projections"] = proj
    out["_ctx_mean"] = float(np.mean(getattr(wl, "lens", [0])))
    # graphs that hold NCCL calls go before the process group does
    if hasattr(wl, "sess"):
        wl.sess.graph = None
        if getattr(wl.sess, "peer", None) is not None:
            gpu.device_synchronize()
            ranks.barrier()   # no peer still writes into the slots
            wl.sess.close()
    if getattr(wl, "tp", None) is not None:
        wl.tp.close()         # NCCL communicator, on every rank
    import gc
    gc.collect()
    gpu.device_synchronize()
    return out


def reference_arm(args, ranks, cores):
    """Rank 0 times the oracle (the reference's math in numpy) on the host."""
    if ranks.rank != 0:
        return None
    if args.workload == "gqa":
        import multiprocessing as mp
        wl = GQAWorkload(ranks, 0, 0, copies=0)
        with mp.get_context("spawn").Pool(cores) as pool:
            vals, sample = [], ""
            for i in range(args.warmup + args.steps):
                v, sample = gqa_cpu_baseline(cores, pool, budget_s=2.0)
                if i >= args.warmup:
                    vals.append(v)
        value = statistics.median(vals)
        cfg = wl.config()
        scaling = wl.scaling
    elif args.workload == "llama3b_tp":
        value, sample = llama_cpu_sample(LlamaTPWorkload.ctx, max(args.steps, 3))
        cfg = {"workload": "cfg5 Llama-3.2-3B long-context greedy decode, KV-head TP",
               "model": LlamaTPWorkload.model, "batch": 8, "ctx": LlamaTPWorkload.ctx}
        scaling = "strong"
    elif args.workload == "gpt2":
        value, sample = gpt2_cpu_sample(max(args.steps, 3))
        cfg = {"workload": "cfg1 GPT-2 small fp32 greedy decode, batch 1",
               "model": "GPT-2 small (124M)", "batch": 1, "prompt": 32}
        scaling = "weak"
    elif args.workload == "smol135m":
        value, sample = llama_cpu_sample(640, max(args.steps, 3),
                                         model=SmolDecodeWorkload.model)
        cfg = {"workload": "cfg3 SmolLM2-135M batched greedy decode",
               "model": SmolDecodeWorkload.model, "batch": 32, "ctx": 640}
        scaling = "weak"
    else:
        from triton_llm import shard
        lens = shard.ragged_lengths(64, LlamaDecodeWorkload.lo, LlamaDecodeWorkload.hi,
                                    LlamaDecodeWorkload.len_seed)
        value, sample = llama_cpu_sample(int(lens.mean()), max(args.steps, 3))
        weak = args.workload == "llama3b_weak"
        cfg = {"workload": "cfg4 Llama-3.2-3B ragged-batch greedy decode",
               "model": LlamaDecodeWorkload.model,
               "global_batch": 64 * ranks.world if weak else 64,
               "ctx": "U[1024,8192] seed 4"}
        scaling = "weak" if weak else "strong"
    return {"impl": "reference", "metric": METRIC, "value": round(value, 4),
            "unit": "tokens/s", "n_gpus": ranks.world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, BASELINE config shapes)", "config": cfg,
            "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s",
                             "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "tokens/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="llama3b", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--act", default="split", choices=["bfloat16", "split"],
                    help="projection input format of the bf16 path (hi + lo planes, "
                         "the default, or one bf16 plane)")
    args = ap.parse_args()
    LlamaDecodeWorkload.act = args.act
    LlamaTPWorkload.act = args.act
    ProjLlamaLayerWorkload.planes = 2 if args.act == "split" else 1
    args.warmup = max(args.warmup, 3)

    ranks = Ranks()
    cores = len(os.sched_getaffinity(0))

    if args.impl == "reference":
        line = reference_arm(args, ranks, cores)
        if line is not None:
            print(json.dumps(line), flush=True)
        ranks.close()
        return

    pool = None
    want_cpu = ranks.world == 1 and not args.no_cpu_baseline
    if want_cpu and args.workload == "gqa":
        # spawn the CPU-baseline workers before the first GPU call
        import multiprocessing as mp
        pool = mp.get_context("spawn").Pool(cores)
    out = run_b200(args, ranks)
    ctx = out.pop("_ctx_mean")
    if want_cpu:
        res = cpu_baseline(args.workload, cores, 5, pool, ctx)
        if pool is not None:
            pool.close()
        if res is not None:
            v, sample = res
            out["cpu_baseline"] = {"value": round(v, 4), "unit": "tokens/s",
                                   "cores": cores, "kind": "port", "sample": sample}
    if ranks.rank == 0:
        print(json.dumps(out), flush=True)
    ranks.close()


if __name__ == "__main__":
    main()
