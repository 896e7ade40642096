"""bench.py's reference arm on the host (no GPU): the JSON line the driver
reads, and the multi-rank rule (rank 0 alone runs and prints; the other
ranks exit 0 without work)."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
BENCH = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--workload", "gpt2",
         "--steps", "1", "--warmup", "3"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check_line(line: dict):
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
              "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference"
    assert line["warmup"] >= 3 and line["steps"] == 1
    assert line["value"] > 0 and line["unit"] == "tokens/s"
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"].startswith("cfg1")


def test_reference_arm_prints_one_line():
    out = subprocess.run(BENCH, cwd=REPO, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    _check_line(json.loads(lines[0]))


def test_reference_arm_two_ranks_rank0_only():
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2",
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        procs.append(subprocess.Popen(BENCH + ["--gpus", "2"], cwd=REPO, env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                      text=True))
    outs = []
    for p in procs:
        try:
            so, se = p.communicate(timeout=300)
        finally:
            if p.poll() is None:
                p.kill()
        outs.append((p.returncode, so, se))
    for rc, so, se in outs:
        assert rc == 0, se[-2000:]
    rank0 = [ln for ln in outs[0][1].splitlines() if ln.strip()]
    assert len(rank0) == 1
    _check_line(json.loads(rank0[0]))
    assert not outs[1][1].strip()   # rank 1 prints nothing


def test_projection_kernel_labels(monkeypatch):
    """The roofline line names the kernel tllm_linear picks for each
    projection (the skinny kernel for small decode batches on small
    matrices, tcgen05 otherwise, fp32 CUDA cores for fp32 weights)."""
    for p in (REPO / "triton-llm_b200", REPO):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    import bench
    from triton_llm.kernels.linear import kernel_name
    monkeypatch.delenv("TLLM_SKINNY_MAX_M", raising=False)
    monkeypatch.delenv("TLLM_SKINNY_MAX_MB", raising=False)
    smol = [(32, 960, 576), (32, 576, 576), (32, 3072, 576), (32, 576, 1536), (32, 49152, 576)]
    llama = [(64, 5120, 3072), (64, 3072, 3072), (64, 16384, 3072), (64, 3072, 8192),
             (64, 128256, 3072)]
    assert bench.projection_kernels(smol, False) == (
        "linear_mma_kernel (qkv+rope+append, o, gate/up+swiglu, down) + "
        "linear_tc_kernel (lm_head)")
    assert bench.projection_kernels(llama, False) == (
        "linear_tc_kernel (qkv+rope+append, o, gate/up+swiglu, down, lm_head)")
    assert "mlp_kernel" in bench.projection_kernels(llama, True)
    assert kernel_name(8, 4096, 1024) == "linear_mma_kernel"        # exactly 8 MiB
    assert kernel_name(8, 4096, 1088) == "linear_tc_kernel"         # above it
    assert kernel_name(33, 576, 576) == "linear_tc_kernel"
    assert kernel_name(8, 576, 576, scatter=True) == "linear_tc_kernel"
    assert kernel_name(1, 768, 768, bf16=False) == "linear_f32_kernel"
    monkeypatch.setenv("TLLM_SKINNY_MAX_M", "0")
    assert kernel_name(1, 576, 576) == "linear_tc_kernel"
    monkeypatch.setenv("TLLM_SKINNY_MAX_M", "32")
    monkeypatch.setenv("TLLM_SKINNY_MAX_MB", "1")
    assert kernel_name(32, 576, 576) == "linear_mma_kernel"         # 0.63 MiB
    assert kernel_name(32, 3072, 576) == "linear_tc_kernel"         # 3.4 MiB
