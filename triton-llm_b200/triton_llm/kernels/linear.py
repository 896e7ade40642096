"""Projection weights and the fused GEMM (tllm_linear).

``Linear`` holds one projection on the device in the layout the kernels
read: HF (out, in) rows, bf16 or fp32, with the row order the epilogue
expects -- gate/up rows interleaved in blocks of 8 for SwiGLU, and each
q/k/v head stored as (8b..8b+7, D/2+8b..D/2+8b+7) blocks so the RoPE pair
(d, d + D/2) of the reference's rotate-half (triton_llm/kernels/rope.py:
49-66) lands in one thread. ``LinearWorkspace`` holds the split-K scratch
shared by every projection of a model.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from triton_llm import gpu, _lib


def swiglu_rows(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """(F, K) gate and up -> (2F, K) interleaved in blocks of 8 rows."""
    F, K = gate.shape
    if F % 8:
        raise ValueError(f"intermediate size {F} must be a multiple of 8")
    g = gate.reshape(F // 8, 8, K)
    u = up.reshape(F // 8, 8, K)
    return np.ascontiguousarray(np.stack([g, u], axis=1).reshape(2 * F, K))


def head_row_order(D: int) -> np.ndarray:
    """Permutation of one head's D rows: (8b..8b+7, D/2+8b..D/2+8b+7)."""
    if D % 16:
        raise ValueError(f"head_dim {D} must be a multiple of 16")
    order = []
    for b in range(D // 16):
        order += list(range(8 * b, 8 * b + 8))
        order += list(range(D // 2 + 8 * b, D // 2 + 8 * b + 8))
    return np.array(order, np.int64)


def qkv_rows(wq, wk, wv, D, bq=None, bk=None, bv=None):
    """Stack q, k, v heads (HF (out, in)) with the per-head RoPE row order."""
    w = np.concatenate([wq, wk, wv], axis=0)
    n_heads = w.shape[0] // D
    perm = (np.arange(n_heads)[:, None] * D + head_row_order(D)[None, :]).reshape(-1)
    w = np.ascontiguousarray(w[perm])
    b = None
    if bq is not None:
        b = np.ascontiguousarray(np.concatenate([bq, bk, bv])[perm], np.float32)
    return w, b


TILE_N, TILE_K = 128, 64


def tile_bf16(bits: np.ndarray) -> np.ndarray:
    """(N, K) bf16 bits -> the TLLM_BF16_TILED layout: contiguous 128 x 64
    tiles in (row tile, k chunk) order, N padded to 128 with zero rows."""
    N, K = bits.shape
    if K % TILE_K:
        raise ValueError(f"bf16 weights need K % {TILE_K} == 0 (K={K})")
    n_pad = -(-N // TILE_N) * TILE_N
    padded = np.zeros((n_pad, K), np.uint16)
    padded[:N] = bits
    t = padded.reshape(n_pad // TILE_N, TILE_N, K // TILE_K, TILE_K).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(t).reshape(-1)


def untile_bf16(flat: np.ndarray, N: int, K: int) -> np.ndarray:
    n_pad = -(-N // TILE_N) * TILE_N
    t = flat.reshape(n_pad // TILE_N, K // TILE_K, TILE_N, TILE_K).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(t).reshape(n_pad, K)[:N]


class Linear:
    """A projection y = x W^T (+ b) with W (N, K) on the device.

    bf16 weights are stored tiled (TLLM_BF16_TILED: every 128 x 64 tile the
    tensor-core projection streams is one contiguous 16 KB block); fp32
    weights stay row-major (N, K).
    """

    # TLLM_TILE_WEIGHTS=0 keeps bf16 weights row-major (comparisons)
    tiled_default = os.environ.get("TLLM_TILE_WEIGHTS", "1") != "0"

    def __init__(self, w: np.ndarray, dtype: str = "bfloat16", bias=None):
        w = np.ascontiguousarray(w, np.float32)
        self.N, self.K = w.shape
        self.bf16 = dtype in ("bfloat16", "bf16")
        self.tiled = self.bf16 and self.tiled_default
        if self.bf16:
            bits = gpu.f32_to_bf16_bits(w)
            if self.tiled:
                flat = tile_bf16(bits)
            else:
                if self.K % TILE_K:
                    raise ValueError(f"bf16 weights need K % {TILE_K} == 0 (K={self.K})")
                flat = bits.reshape(-1)
            self.w = gpu.allocate(flat.shape, gpu.BFLOAT16)
            self.w.from_numpy(flat)
        else:
            self.w = gpu.to_device(w)
        self.b = gpu.to_device(np.ascontiguousarray(bias, np.float32)) if bias is not None else None

    @classmethod
    def empty_bf16(cls, N: int, K: int):
        """Uninitialised bf16 weights (filled on the device)."""
        if K % TILE_K:
            raise ValueError(f"bf16 weights need K % {TILE_K} == 0 (K={K})")
        obj = cls.__new__(cls)
        obj.N, obj.K, obj.bf16, obj.b = int(N), int(K), True, None
        obj.tiled = cls.tiled_default
        n_pad = -(-obj.N // TILE_N) * TILE_N if obj.tiled else obj.N
        obj.w = gpu.allocate((n_pad * obj.K,), gpu.BFLOAT16)
        return obj

    @property
    def dtype(self):
        if not self.bf16:
            return _lib.F32
        return _lib.BF16_TILED if self.tiled else _lib.BF16

    def to_numpy(self) -> np.ndarray:
        """The (N, K) weights as fp32 on the host."""
        if not self.bf16:
            return self.w.to_numpy()
        flat = self.w.to_numpy()
        bits = untile_bf16(flat, self.N, self.K) if self.tiled else flat.reshape(self.N, self.K)
        return gpu.bf16_bits_to_f32(bits)


class LinearWorkspace:
    """Split-K scratch of tllm_linear, sized for the largest (M, N, K)."""

    def __init__(self, shapes):
        pb_max, cb_max = 0, 0
        for (M, N, K) in shapes:
            pb, cb = ctypes.c_size_t(), ctypes.c_size_t()
            _lib.call("tllm_linear_workspace", int(M), int(N), int(K),
                      ctypes.byref(pb), ctypes.byref(cb))
            pb_max = max(pb_max, pb.value)
            cb_max = max(cb_max, cb.value)
        self.partial_bytes = pb_max
        self.partial = gpu.allocate((max(pb_max // 4, 1),), np.float32)
        self.counters = gpu.zeros((max(cb_max // 4, 1),), np.int32)


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name, "")
    try:
        return int(v) if v else default
    except ValueError:
        return 0   # like atoi on the C side


def kernel_name(M: int, N: int, K: int, bf16: bool = True, scatter: bool = False) -> str:
    """The kernel ``tllm_linear`` runs for an (M, N, K) projection, by the
    C side's rule: fp32 weights -> linear_f32_kernel; bf16 weights with at
    most TLLM_SKINNY_MAX_M (32) rows on a matrix of at most
    TLLM_SKINNY_MAX_MB (8) MiB, and not SCATTER -> linear_mma_kernel;
    otherwise linear_tc_kernel."""
    if not bf16:
        return "linear_f32_kernel"
    max_m = min(max(_env_int("TLLM_SKINNY_MAX_M", 32), 0), 32)
    max_bytes = max(_env_int("TLLM_SKINNY_MAX_MB", 8), 0) << 20
    if not scatter and M <= max_m and N * K * 2 <= max_bytes:
        return "linear_mma_kernel"
    return "linear_tc_kernel"


def plan(M: int, N: int, K: int, planes: int = 1) -> dict:
    """Launch plan of the bf16 tensor-core path (tllm_linear_plan) for
    activations with 1 (TLLM_BF16) or 2 (TLLM_SPLIT) planes."""
    arr = (ctypes.c_int * 8)()
    _lib.call("tllm_linear_plan", int(M), int(N), int(K),
              _lib.SPLIT if planes == 2 else _lib.BF16, arr)
    keys = ("tile_m", "m_tiles", "n_tiles", "splits", "weight_stages", "smem_bytes",
            "act_stages", "resident_ctas")
    return dict(zip(keys, list(arr)))


def to_split(x_dev, M=None, out=None, planes=2):
    """fp32 (rows, K) -> operand-format buffer (TLLM_SPLIT by default)."""
    rows, K = int(x_dev.shape[0]), int(x_dev.shape[-1])
    M = rows if M is None else int(M)
    if out is None:
        out = gpu.act_empty(rows, K, planes)
    _lib.call("tllm_split_bf16", x_dev.ptr, out.ptr,
              _lib.SPLIT if out.shape[0] == 2 else _lib.BF16, M, K, int(out.shape[1]),
              None)
    return out


def fold_parts(M: int, N: int, K: int) -> int:
    """Partial sums per row a folded-norm producer (M, N, K) writes."""
    out = ctypes.c_int(0)
    _lib.call("tllm_linear_fold_parts", int(M), int(N), int(K), ctypes.byref(out))
    return out.value


class FoldedNorm:
    """An RMSNorm folded into the projections around it (tllm_norm_fold):
    the projection that writes its input (op RESID; ``rows`` rows, K =
    ``producer_k``) also writes ``fx`` = h * ``weight`` in operand format
    and per-column-part sums of squares into ``ss``; the projection that
    reads ``fx`` divides each output row by the row's rms. ``fx`` is an
    operand buffer of at least ``rows`` rows; ``ss`` fp32
    (>= ceil(hidden / 16), >= rows)."""

    def __init__(self, weight, fx, ss, hidden: int, eps: float, rows: int,
                 producer_k: int):
        self.weight, self.fx, self.ss = weight, fx, ss
        self.hidden, self.eps = int(hidden), float(eps)
        self.parts = fold_parts(rows, self.hidden, producer_k)
        if self.parts > int(ss.shape[0]) or rows > int(ss.shape[1]):
            raise ValueError(f"partial-sum buffer {tuple(ss.shape)} too small for "
                             f"{self.parts} parts x {rows} rows")
        self.ld = int(ss.shape[1])

    def producer(self):
        _, dt, plane = gpu.act_args(self.fx)
        return _lib.NormFold(self.weight.data_ptr(), self.fx.data_ptr(), dt, plane,
                             self.ss.data_ptr(), None, 0, self.hidden, self.eps, self.ld)

    def consumer(self):
        return _lib.NormFold(None, None, 0, 0, None, self.ss.data_ptr(), self.parts,
                             self.hidden, self.eps, self.ld)


def linear(x_dev, lin: Linear, out_dev=None, op=_lib.EPI_STORE, resid_dev=None,
           ws: LinearWorkspace | None = None, M=None, ld_out=0, qkv=None,
           p2p=None, stream=None, fold_in: FoldedNorm | None = None,
           fold_out: FoldedNorm | None = None):
    """Run one projection on the first M rows of ``x_dev``.

    ``x_dev``: fp32 (rows, K) or TLLM_SPLIT (2, rows, K) (``gpu.split_empty``);
    bf16 weights take TLLM_SPLIT, and fp32 input is converted first.
    ``out_dev``: fp32 or TLLM_SPLIT. ``qkv`` = dict(cos, sin, row_seq,
    row_pos, q_out, k_cache, v_cache, n_head, n_kv_head, head_dim, lens_out)
    for op QKV. ``p2p``: a ``triton_llm.tp.PeerGroup`` for op SCATTER.
    ``fold_in``: ``x_dev`` is ``fold_in.fx`` (h * norm weight) and the rows
    are divided by their rms; ``fold_out`` (op RESID): also write the next
    norm's ``fx`` and partial sums (``FoldedNorm``).
    """
    split_in = getattr(x_dev, "is_split", False)
    rows = int(x_dev.shape[1] if split_in else x_dev.shape[0])
    M = rows if M is None else int(M)
    K = int(x_dev.shape[-1])
    if K != lin.K:
        raise ValueError(f"linear: x has K={K}, weight has K={lin.K}")
    if lin.bf16 and not split_in:
        x_dev = to_split(x_dev, M)
    xptr, xdt, xplane = gpu.act_args(x_dev)
    optr, odt, oplane = (gpu.act_args(out_dev) if out_dev is not None
                         else (None, _lib.F32, 0))
    q = qkv or {}
    kc = q.get("k_cache")
    fold = None
    if fold_in is not None or fold_out is not None:
        fold = fold_out.producer() if fold_out is not None else _lib.NormFold()
        if fold_in is not None:
            c = fold_in.consumer()
            fold.ss_in, fold.ss_parts, fold.ss_cols = c.ss_in, c.ss_parts, c.ss_cols
            fold.eps = c.eps
            if fold_out is not None and fold_out.ld != fold_in.ld:
                raise ValueError("folded norms on both sides need the same ss row stride")
            fold.ss_ld = c.ss_ld
    _lib.call(
        "tllm_linear_folded", xptr, xdt, xplane, lin.w.ptr, lin.dtype, M, lin.N, lin.K,
        int(op), _lib.ptr(lin.b), optr, odt, oplane, int(ld_out), _lib.ptr(resid_dev),
        _lib.ptr(q.get("cos")), _lib.ptr(q.get("sin")), _lib.ptr(q.get("row_seq")),
        _lib.ptr(q.get("row_pos")), _lib.ptr(q.get("q_out")), _lib.ptr(kc),
        _lib.ptr(q.get("v_cache")),
        _lib.BF16 if (kc is not None and kc.is_bf16) else _lib.F32,
        int(kc.shape[2]) if kc is not None else 0, int(q.get("n_head", 0)),
        int(q.get("n_kv_head", 0)), int(q.get("head_dim", 0)),
        _lib.ptr(q.get("lens_out")), p2p.ctx if p2p is not None else None,
        ws.partial.ptr if ws else None, ws.partial_bytes if ws else 0,
        ws.counters.ptr if ws else None,
        ctypes.byref(fold) if fold is not None else None, stream)
    return out_dev
