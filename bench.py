"""Benchmark of the B200 decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl b200|reference]

Prints ONE JSON line on rank 0. Under torchrun (N > 1) every rank drives
its own GPU; ranks meet only at host barriers (gloo) around the timed
region, and the time reported is the maximum over ranks.

Workloads:
  gqa   config 2: split-KV GQA decode attention, 64 ragged sequences
        (lengths U[128, 2048], seed 1), 9 q / 3 kv heads, head_dim 64, bf16
        KV cache resident in HBM. One step = one attention launch over the
        whole batch; "tokens" = sequences decoded. Each rank runs its own
        batch (weak scaling). Rotating cache copies keep the working set
        above L2.

The reference arm (--impl reference) times the reference's math on the
host cores: the CPU oracle (a numpy restatement of the reference kernels,
oracle/), on the same workload with every host core, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
for _p in (REPO / "triton-llm_b200", REPO, REPO / "tests" / "golden"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "decode tokens/s (whole box)"
FALLBACK_HBM_GBS = 6650.0


# ------------------------------------------------------------------ ranks ----
class Ranks:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ----------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi sampled every 200 ms during the timed region."""

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
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
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


def profiled_traffic(key: str):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu
    summary (profiles/traffic.json), or None."""
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        try:
            d = json.loads(p.read_text()).get(key)
            return d.get("bytes_per_launch") if d else None
        except Exception:
            return None
    return None


# ------------------------------------------------------------- workloads ----
class GQAWorkload:
    """BASELINE config 2 (isolated GQA decode attention)."""

    name = "gqa"
    scaling = "weak"
    dtype = "bf16"
    kernel = "gqa_decode"

    BENCH_COPIES = 6

    def __init__(self, copies=BENCH_COPIES):
        import inputs
        self.B, self.H, self.Hkv, self.D, self.S = 64, 9, 3, 64, 2048
        self.lens, self.q, ks, vs = inputs.cfg2_inputs()
        self.kc = inputs.pack_cache(ks, self.S)
        self.vc = inputs.pack_cache(vs, self.S)
        self.copies = copies
        L = int(self.lens.sum())
        self.kv_bytes = 2 * self.Hkv * L * self.D * 2
        self.bytes_per_step = self.kv_bytes + 2 * self.B * self.H * self.D * 4 + self.B * 4
        self.units_per_step = self.B

    def config(self):
        return {"workload": "cfg2 isolated GQA decode attention",
                "batch": self.B, "n_head": self.H, "n_kv_head": self.Hkv,
                "head_dim": self.D, "kv_lens": "U[128,2048] seed 1",
                "sum_kv_len": int(self.lens.sum()),
                "kv_dtype": "bf16", "kv_layout": "(B, n_kv, 2048, d) prealloc",
                "timed": "K launches replayed as one CUDA graph",
                "l2": f"{self.BENCH_COPIES} rotating cache copies "
                      f"({self.BENCH_COPIES * self.kv_bytes / 1e6:.0f} MB touched > 126 MB L2)"}

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
        # pinned host buffers for the end-to-end leg
        self.q_host = gpu.pinned_empty(self.q.shape, np.float32)
        self.q_host[...] = self.q
        self.l_host = gpu.pinned_empty(self.lens.shape, np.int32)
        self.l_host[...] = self.lens
        self.o_host = gpu.pinned_empty(self.q.shape, np.float32)
        self.h2d = self.q.nbytes + self.lens.nbytes
        self.d2h = self.q.nbytes

    def step(self, i):
        from triton_llm.kernels import gqa_decode
        c = i % self.copies
        gqa_decode(self.qd, self.kd[c], self.vd[c], self.ld, self.od,
                   max_len=self.S, workspace=self.ws)
        return 1  # kernel launches

    def step_e2e(self, i):
        g = self.gpu
        g.copy_h2d_async(self.qd, self.q_host)
        g.copy_h2d_async(self.ld, self.l_host)
        n = self.step(i)
        g.copy_d2h_async(self.o_host, self.od)
        g.stream_synchronize()
        return n

    def check(self):
        """Result of the last step vs the oracle on the first sequences."""
        from oracle import ops
        out = self.od.to_numpy()
        n = 4
        ref = ops.gqa_decode(self.q[:n], self.kc[:n], self.vc[:n], self.lens[:n])
        return float(np.abs(out[:n] - ref).max())

    # ---- CPU baseline: the oracle (numpy restatement) on a sample ----
    def cpu_sample(self, nseq):
        idx = np.arange(nseq) % self.B
        return idx

    def cpu_run(self, idx):
        from oracle import ops
        ops.gqa_decode(self.q[idx], self.kc[idx], self.vc[idx], self.lens[idx])
        return len(idx)


WORKLOADS = {"gqa": GQAWorkload}


# ----------------------------------------------------------- CPU baseline ----
_worker_wl: dict = {}


def _make_cpu_workload(name):
    return GQAWorkload(copies=0) if name == "gqa" else WORKLOADS[name]()


def _cpu_worker(args):
    """Pool worker: run the oracle on a list of sample indices."""
    name, idx = args
    if name not in _worker_wl:
        _worker_wl[name] = _make_cpu_workload(name)
    wl = _worker_wl[name]
    t = time.perf_counter()
    n = wl.cpu_run(np.asarray(idx, dtype=np.int64))
    return n, time.perf_counter() - t


def cpu_baseline(name, cores, pool, budget_s=15.0):
    """Time the oracle (numpy restatement of the reference) on a bounded
    sample spread over `cores` worker processes. Returns (units/s, text)."""
    wl = _make_cpu_workload(name)
    # warm every worker (input generation) and calibrate one unit
    warm = pool.map(_cpu_worker, [(name, [0])] * cores)
    per = max(min(r[1] for r in warm), 1e-4)
    per_worker = max(1, int(budget_s / per))
    nseq = min(per_worker * cores, 8 * wl.B)
    idx = wl.cpu_sample(nseq)
    chunks = [idx[i::cores].tolist() for i in range(cores)]
    t = time.perf_counter()
    res = pool.map(_cpu_worker, [(name, c) for c in chunks if c])
    dt = time.perf_counter() - t
    done = sum(r[0] for r in res)
    return done / dt, f"oracle on {done} sequences over {cores} processes ({dt:.1f} s)"


# ------------------------------------------------------------------ main ----
def run_b200(args, ranks):
    from triton_llm import gpu
    gpu.set_device(ranks.local)
    gpu.device_error(reset=True)
    wl = WORKLOADS[args.workload]()
    wl.setup()
    gpu.device_synchronize()

    # warm-up
    for i in range(args.warmup):
        wl.step(i)
    gpu.device_synchronize()

    # The K timed steps are captured once as a CUDA graph (the decode loop
    # of a server is replayed the same way), so host launch cost stays off
    # the device timeline; the graph is replayed once untimed first.
    launches = 0
    graph = gpu.Graph()
    with graph:
        for i in range(args.steps):
            launches += wl.step(args.warmup + i)
    graph.launch()
    gpu.device_synchronize()

    # timed region (device events on the library stream), clocks sampled
    clocks = ClockSampler(ranks.local)
    clocks.start()
    ranks.barrier()
    gpu.device_synchronize()
    e0, e1 = gpu.Event(), gpu.Event()
    e0.record()
    graph.launch()
    e1.record()
    gpu.device_synchronize()
    ranks.barrier()
    ms = e0.elapsed_ms(e1)
    clk = clocks.stop()
    ms_max = ranks.max(ms)

    # end-to-end leg: host buffers, copies inside the timed region
    for i in range(2):
        wl.step_e2e(i)
    ranks.barrier()
    gpu.device_synchronize()
    t0, t1 = gpu.Event(), gpu.Event()
    t0.record()
    for i in range(args.steps):
        wl.step_e2e(i)
    t1.record()
    gpu.device_synchronize()
    ranks.barrier()
    e2e_ms = ranks.max(t0.elapsed_ms(t1))

    err = wl.check()
    dev_err = gpu.device_error()
    units = ranks.sum(wl.units_per_step * args.steps)
    value = units / (ms_max / 1e3)
    e2e_value = units / (e2e_ms / 1e3)

    peak, peak_kind = measured_peaks()
    per_launch_ms = ms / args.steps  # this rank, dominant kernel only
    achieved = wl.bytes_per_step / (per_launch_ms / 1e3) / 1e9
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": ranks.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 5),
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
        "dtype": wl.dtype, "data": "synthetic (seeded, BASELINE config inputs)",
        "config": wl.config(),
        "parallelism": f"dp{ranks.world} (independent replicas, no collective)",
        "roofline": {"bound": "hbm", "kernel": wl.kernel,
                     "achieved": round(achieved, 1), "peak": peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "algorithmic_bytes_per_launch": wl.bytes_per_step,
                     "traffic": profiled_traffic(wl.name)},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h},
        "gpu_launches": launches,
        "clocks": clk,
        "check": {"max_abs_err_vs_oracle": err, "device_error": dev_err},
    }
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="gqa", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    ranks = Ranks()
    cores = len(os.sched_getaffinity(0))

    if args.impl == "reference":
        if ranks.rank != 0:
            ranks.close()
            return
        import multiprocessing as mp
        ctx = mp.get_context("spawn")
        with ctx.Pool(cores) as pool:
            wl = _make_cpu_workload(args.workload)
            vals = []
            for i in range(args.warmup + args.steps):
                v, sample = cpu_baseline(args.workload, cores, pool, budget_s=2.0)
                if i >= args.warmup:
                    vals.append(v)
        value = statistics.median(vals)
        line = {"impl": "reference", "metric": METRIC, "value": round(value, 3),
                "unit": "tokens/s", "n_gpus": ranks.world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True,
                "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, BASELINE config inputs)",
                "config": wl.config(),
                "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s",
                                 "cores": cores, "kind": "port",
                                 "sample": sample + " per step; numpy restatement "
                                 "of the reference kernels (oracle/)"},
                "e2e": {"value": round(value, 3), "unit": "tokens/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        ranks.close()
        return

    pool = None
    if ranks.world == 1 and not args.no_cpu_baseline:
        # spawn the CPU-baseline workers before the first GPU call
        import multiprocessing as mp
        pool = mp.get_context("spawn").Pool(cores)
    out = run_b200(args, ranks)
    if pool is not None:
        v, sample = cpu_baseline(args.workload, cores, pool)
        pool.close()
        out["cpu_baseline"] = {"value": round(v, 3), "unit": "tokens/s",
                               "cores": cores, "kind": "port",
                               "sample": sample + "; numpy restatement of the "
                               "reference kernels (oracle/)"}
    if ranks.rank == 0:
        print(json.dumps(out), flush=True)
    ranks.close()


if __name__ == "__main__":
    main()
