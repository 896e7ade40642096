"""Tensor parallelism by KV head (config 5).

* CPU, world size 2 (gloo): the engine's sharding (``shard_llama_layer``)
  plus an all-reduce of the o / down partial sums reproduces the oracle's
  full forward pass -- the TP math, independent of the GPU.
* GPU, 2 ranks (skipped with fewer than 2 GPUs): the TP engine on the
  Llama-3.2-3B 2-layer slice against the reference's own logits and tokens,
  run as two plain processes over the package's rendezvous and NCCL binding
  (no torch in them).
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import inputs

REPO = Path(__file__).resolve().parent.parent
SMALL = inputs.LlamaShape(100, 128, 2, 8, 4, 256, 64)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp_forward_rank(rank, world, port, out_q):
    import torch
    import torch.distributed as dist
    from oracle import ops
    from triton_llm import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shp = SMALL
    w = inputs.llama_weights(shp, 3)
    n, H, Hkv, F = shp.hidden_size, shp.num_attention_heads, shp.num_key_value_heads, shp.intermediate_size
    D = n // H
    ids = np.array([5, 17, 3, 99, 42, 7])
    T = len(ids)
    cos, sin = ops.precompute_cos_sin(shp.max_position_embeddings, D, shp.rope_theta)
    h = np.asarray(w["model.embed_tokens.weight"], np.float32)[ids]
    Hl, Hkvl, _ = shard.tp_dims(H, Hkv, F, world)

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
        dist.all_reduce(t)
        return t.numpy()

    for i in range(shp.num_hidden_layers):
        lw = shard.shard_llama_layer(w, f"model.layers.{i}.", D, H, Hkv, F, rank, world)
        x = ops.rms_norm(h, lw["ln1"], shp.rms_norm_eps)
        q = ops.gemm(x, lw["q"].T).reshape(T, Hl, D).transpose(1, 0, 2).reshape(-1, D)
        k = ops.gemm(x, lw["k"].T).reshape(T, Hkvl, D).transpose(1, 0, 2).reshape(-1, D)
        v = ops.gemm(x, lw["v"].T).reshape(T, Hkvl, D).transpose(1, 0, 2).reshape(-1, D)
        q = ops.apply_rope(q, cos, sin, T, 0)
        k = ops.apply_rope(k, cos, sin, T, 0)
        o = ops.gqa_attention(q, k, v, Hl, Hkvl, causal=True)
        o = o.reshape(Hl, T, D).transpose(1, 0, 2).reshape(T, Hl * D)
        h = h + allreduce(ops.gemm(o, lw["o"].T))
        x = ops.rms_norm(h, lw["ln2"], shp.rms_norm_eps)
        act = ops.swiglu(ops.gemm(x, lw["gate"].T), ops.gemm(x, lw["up"].T))
        h = h + allreduce(ops.gemm(act, lw["down"].T))
    x = ops.rms_norm(h, np.asarray(w["model.norm.weight"], np.float32), shp.rms_norm_eps)
    logits = ops.gemm(x, np.asarray(w["model.embed_tokens.weight"], np.float32).T)
    dist.destroy_process_group()
    if rank == 0:
        out_q.put(logits)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_sharding_matches_full_model(world):
    import multiprocessing as mp
    from oracle.models import SmolLM2Oracle
    from smollm2_triton import SmolLM2Config
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_forward_rank, args=(r, world, port, qu))
             for r in range(world)]
    for p in procs:
        p.start()
    got = qu.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = inputs.llama_weights(SMALL, 3)
    o = SmolLM2Oracle(SmolLM2Config(**SMALL.config_kwargs()), w)
    o.init_cache(16)
    ref = o.forward_cached(np.array([[5, 17, 3, 99, 42, 7]]))[0]
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_tp_dims_reject_uneven():
    from triton_llm import shard
    assert shard.tp_dims(24, 8, 8192, 8) == (3, 1, 1024)
    with pytest.raises(ValueError):
        shard.tp_dims(9, 3, 1536, 2)


_GPU_TP = r"""
import os, sys, json
import numpy as np
sys.path[:0] = [os.path.join(os.getcwd(), p) for p in ("triton-llm_b200", ".", "tests/golden")]
import inputs
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
from triton_llm import gpu
from triton_llm.rendezvous import Rendezvous
from triton_llm.tp import TPGroup
from smollm2_triton import SmolLM2Config
from smollm2_triton.engine import LlamaSession, LlamaWeights
assert "torch" not in sys.modules
rdzv = Rendezvous.from_env(timeout=300)
tp = TPGroup(rank, world, rank, rdzv=rdzv, timeout_ms=60000)
g = np.load("tests/golden/llama3b_2l_slice.npz")
w = inputs.round_linear_weights_bf16(inputs.llama_weights(inputs.LLAMA3B_2L, 0))
cfg = SmolLM2Config(**inputs.LLAMA3B_2L.config_kwargs())
wts = LlamaWeights(cfg, w, "bfloat16", max_pos=64, tp_rank=rank, tp_size=world)
prompt = g["tokens"][:4].tolist()
sess = LlamaSession(wts, 1, 8, kv_dtype="float32", act_dtype="split", tp=tp)
logits = [sess.prefill([prompt])[0]]
toks = prompt + [int(np.argmax(logits[0]))]
sess.decode_step(sample=True)
gpu.device_synchronize()
logits.append(sess.logits.to_numpy()[0])
toks.append(int(sess.ids.to_numpy()[0]))
err = float(np.abs(np.stack(logits) - g["logits"]).max())
# graph-captured steps: fused peer all-reduce (default) against NCCL
runs = []
for p2p in (True, False):
    s2 = LlamaSession(wts, 2, 16, kv_dtype="float32", act_dtype="split", tp=tp, p2p=p2p)
    s2.prefill([prompt, prompt[:3]])
    s2.capture()
    tk, lg = [], []
    for _ in range(4):
        s2.step()
        gpu.device_synchronize()
        tk.append(s2.ids.to_numpy().tolist())
        lg.append(s2.logits.to_numpy())
    runs.append((tk, np.stack(lg)))
    s2.graph = None
    tp.barrier()
    s2.close()
same = runs[0][0] == runs[1][0]
p2p_err = float(np.abs(runs[0][1] - runs[1][1]).max())
healthy = tp.healthy()
if rank == 0:
    print(json.dumps({"tokens": toks, "want": g["tokens"].tolist(), "err": err,
                      "p2p_same_tokens": same, "p2p_err": p2p_err, "healthy": healthy,
                      "dev_err": gpu.device_error(), "torch": "torch" in sys.modules}))
tp.barrier()
sess.close()
del sess
tp.close()
rdzv.close()
"""


def _gpu_count():
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=30)
        return len([l for l in out.stdout.splitlines() if l.startswith("GPU")])
    except Exception:
        return 0


def _launch_ranks(script, world, timeout_s=600):
    """One process per GPU (rank r on device r), meeting over the package's
    TCP rendezvous; no torchrun and no torch.distributed. NVLS is off (the
    peer path uses plain peer loads and stores; NCCL must not bind NVLink
    multicast objects in a test)."""
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", TLLM_RDZV_PORT=str(port),
                   NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen(
            ["timeout", "-k", "30", str(timeout_s), sys.executable, str(script)],
            cwd=str(REPO), env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
            text=True))
    outs = [p.communicate() for p in procs]
    return [p.returncode for p in procs], outs


@pytest.mark.gpu
def test_tp2_engine_matches_reference(tmp_path):
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    import json
    script = tmp_path / "tp2.py"
    script.write_text(_GPU_TP)
    rcs, outs = _launch_ranks(script, 2)
    assert rcs == [0, 0], "\n".join(o[0][-2000:] + o[1][-4000:] for o in outs)
    line = [ln for ln in outs[0][0].splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    assert d["tokens"] == d["want"], d
    assert d["err"] < 1e-3, d
    assert d["p2p_same_tokens"] and d["p2p_err"] < 1e-3, d
    assert d["dev_err"] == 0 and d["healthy"], d
    assert not d["torch"], "the tensor-parallel path imported torch"
