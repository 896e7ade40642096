"""Parity check of one decode-kernel path, run in a child process.

The decode entry point picks its kernel once per process (the tensor-core
kernel for bf16 caches at head_dim 64/128, or the CUDA-core kernel with
TLLM_GQA_NO_MMA=1), so tests/test_attention_decode_gpu.py runs this script
under each setting. Exits non-zero on a mismatch.
"""

import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
for p in (REPO / "triton-llm_b200", REPO, REPO / "tests" / "golden"):
    sys.path.insert(0, str(p))

import numpy as np  # noqa: E402

import inputs  # noqa: E402
from oracle import ops  # noqa: E402
from triton_llm import gpu  # noqa: E402
from triton_llm.kernels import gqa_decode  # noqa: E402

F32 = np.float32


def run(H, Hkv, D, lens, S, seed):
    rng = np.random.default_rng(seed)
    B = len(lens)
    q = inputs.bf16_round(rng.standard_normal((B, H, D), dtype=F32))
    kc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    vc = inputs.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=F32))
    for b, L in enumerate(lens):
        kc[b, :, L:] = np.nan
        vc[b, :, L:] = np.inf
    od = gpu.allocate((B, H, D), np.float32)
    gqa_decode(gpu.to_device(q), gpu.to_device_bf16(kc), gpu.to_device_bf16(vc),
               gpu.to_device(np.asarray(lens, np.int32)), od, max_len=int(max(lens)))
    out = od.to_numpy()
    ref = ops.gqa_decode(q, kc, vc, np.asarray(lens))
    err = float(np.abs(out - ref).max())
    return err


def main():
    gpu.device_error(reset=True)
    worst = 0.0
    lens = [0, 1, 63, 64, 65, 127, 300, 1023, 1100, 2048]
    for (H, Hkv, D) in ((9, 3, 64), (24, 8, 128), (12, 12, 64), (32, 2, 128)):
        worst = max(worst, run(H, Hkv, D, lens, 2048, H * 7 + D))
    # a small ragged batch at config-4 geometry (splits far shorter than
    # max_len for most rows)
    rng = np.random.default_rng(11)
    lens8 = sorted(rng.integers(512, 4096, 8).tolist())
    worst = max(worst, run(24, 8, 128, lens8, 4096, 5))
    lens_c2, q, ks, vs = inputs.cfg2_inputs(batch=32)
    kc = inputs.pack_cache(ks, 2048)
    vc = inputs.pack_cache(vs, 2048)
    od = gpu.allocate(q.shape, np.float32)
    gqa_decode(gpu.to_device(q), gpu.to_device_bf16(kc), gpu.to_device_bf16(vc),
               gpu.to_device(lens_c2), od, max_len=2048)
    worst = max(worst, float(np.abs(od.to_numpy() - ops.gqa_decode(q, kc, vc, lens_c2)).max()))
    dev = gpu.device_error()
    print(f"max_abs_err={worst:.3e} device_error={dev}")
    sys.exit(0 if (worst < 1e-4 and dev == 0) else 1)


if __name__ == "__main__":
    main()
