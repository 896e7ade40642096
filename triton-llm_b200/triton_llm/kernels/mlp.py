"""The decode MLP half of a Llama-style layer in one launch (tllm_mlp).

h += attn . Wo^T; x = RMSNorm(h) * ln_w; act = silu(x Wg^T) * (x Wu^T);
h += act . Wd^T -- the o projection, the norm before the MLP, gate/up with
SwiGLU and down, which smollm2_triton/model.py:344-357 runs as separate
kernels. One persistent cooperative launch streams the three weight
matrices through every SM without a break.
"""

from __future__ import annotations

import ctypes

import numpy as np

from triton_llm import gpu, _lib

MAX_ROWS = 64


class MlpWorkspace:
    """Counters and split-K partials of tllm_mlp for up to ``rows`` rows."""

    def __init__(self, rows: int, attn_dim: int, hidden: int, ffn: int):
        n = ctypes.c_size_t()
        _lib.call("tllm_mlp_workspace", int(rows), int(attn_dim), int(hidden), int(ffn),
                  ctypes.byref(n))
        self.rows, self.attn_dim, self.hidden, self.ffn = rows, attn_dim, hidden, ffn
        self.nbytes = n.value
        self.buf = gpu.zeros((max(self.nbytes, 1),), np.uint8)

    def reset(self):
        """Zero the counters again (needed after a call that set the device
        error word: a bounded wait that gave up leaves them mid-count)."""
        gpu.memset(self.buf, 0)


def supported(rows: int, attn_dim: int, hidden: int, ffn: int) -> bool:
    return (0 < rows <= MAX_ROWS and hidden % 128 == 0 and attn_dim % 64 == 0
            and ffn % 64 == 0)


def mlp_block(attn, wo, h, ln_w, x, wgu, act, wdown, M: int, eps: float,
              ws: MlpWorkspace, stream=None):
    """Run the block on rows 0..M-1. ``attn``, ``x``, ``act``: one-plane bf16
    operand buffers (``gpu.act_empty(rows, cols, 1)``); weights: tiled bf16
    ``Linear`` objects (``wgu`` with gate/up rows interleaved as for
    ``swiglu_rows``); ``h``: fp32 (rows, hidden), updated in place."""
    for t in (attn, x, act):
        if not getattr(t, "is_split", False) or int(t.shape[0]) != 1:
            raise ValueError("attn, x and act must be one-plane bf16 operand buffers")
    for lin in (wo, wgu, wdown):
        if not (lin.bf16 and lin.tiled):
            raise ValueError("tllm_mlp needs tiled bf16 weights")
    hidden = int(h.shape[-1])
    _lib.call("tllm_mlp", attn.ptr, int(attn.shape[1]), wo.w.ptr, h.ptr, ln_w.ptr,
              float(eps), x.ptr, int(x.shape[1]), wgu.w.ptr, act.ptr, int(act.shape[1]),
              wdown.w.ptr, int(M), int(wo.K), hidden, int(wdown.K), ws.buf.ptr, ws.nbytes,
              stream)
    return h
