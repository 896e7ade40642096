"""ctypes binding of libtllm.so (the sm_100a kernels and device runtime).

The shared library is built in-tree by ``triton-llm_b200/csrc/build.py`` (or
``__graft_entry__.build()``). There is no fallback: if the library or a CUDA
device is missing, every entry point raises. Status codes returned by the C
ABI (include/tllm.h) are mapped onto the exception types the reference uses:

* ``TLLM_ERR_INVALID_ARG`` -> ``ValueError`` (reference kernels raise
  ``ValueError`` for bad shapes, e.g. triton_llm/kernels/attention_gqa.py:189)
* ``TLLM_ERR_NO_DEVICE``   -> ``RuntimeError("No supported GPU runtime found...")``
  (same text as triton_llm/gpu.py:83-86, which callers match on)
* anything else            -> ``RuntimeError("GPU runtime error (cuda): ...")``
  (triton_llm/gpu.py:179-181)
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libtllm.so")

OK = 0
ERR_INVALID_ARG = 1
ERR_CUDA = 2
ERR_UNSUPPORTED = 3
ERR_NO_DEVICE = 4
ERR_NCCL = 5
ERR_TIMEOUT = 6
ERR_INJECTED = 7

F32 = 0
BF16 = 1
I32 = 2
SPLIT = 3   # fp32 values as two bf16 planes (hi, lo): tensor-core operand format
BF16_TILED = 4  # bf16 weights as contiguous 128 x 64 tiles (16 KB per tile)

_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_l = ctypes.c_long
_f = ctypes.c_float
_pvp = ctypes.POINTER(ctypes.c_void_p)
_pi = ctypes.POINTER(ctypes.c_int)
_psz = ctypes.POINTER(ctypes.c_size_t)
_pf = ctypes.POINTER(ctypes.c_float)

# name -> argtypes (restype is always int except tllm_last_error_string)
SIGNATURES: dict[str, list] = {
    "tllm_version": [],
    "tllm_device_count": [_pi],
    "tllm_set_device": [_i],
    "tllm_get_device": [_pi],
    "tllm_get_stream": [_pvp],
    "tllm_malloc": [_pvp, _sz],
    "tllm_free": [_vp],
    "tllm_malloc_static": [_pvp, _sz],
    "tllm_free_static": [_vp],
    "tllm_host_alloc": [_pvp, _sz],
    "tllm_host_free": [_vp],
    "tllm_memcpy_h2d": [_vp, _vp, _sz],
    "tllm_memcpy_d2h": [_vp, _vp, _sz],
    "tllm_memcpy_d2d": [_vp, _vp, _sz],
    "tllm_memcpy_h2d_async": [_vp, _vp, _sz, _vp],
    "tllm_memcpy_d2h_async": [_vp, _vp, _sz, _vp],
    "tllm_memset": [_vp, _i, _sz, _vp],
    "tllm_synchronize": [],
    "tllm_stream_synchronize": [_vp],
    "tllm_device_synchronize": [],
    "tllm_stream_create": [_pvp],
    "tllm_stream_destroy": [_vp],
    "tllm_event_create": [_pvp],
    "tllm_event_destroy": [_vp],
    "tllm_event_record": [_vp, _vp],
    "tllm_event_elapsed_ms": [_vp, _vp, _pf],
    "tllm_stream_wait_event": [_vp, _vp],
    "tllm_device_error": [_pi, _i],
    "tllm_mem_info": [_psz, _psz],
    "tllm_graph_capture_begin": [_vp],
    "tllm_graph_capture_end": [_vp, _pvp],
    "tllm_graph_launch": [_vp, _vp],
    "tllm_graph_destroy": [_vp],
    # attention
    "tllm_gqa_decode_workspace": [_i, _i, _i, _i, _i, _i, _psz, _psz],
    "tllm_gqa_decode": [_vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _i,
                        _f, _vp, _sz, _vp, _vp],
    "tllm_gqa_decode_noalloc": [_vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i,
                                _i, _i, _f, _vp],
    "tllm_gqa_decode_noalloc_error": [_pi, _i],
    "tllm_gqa_prefill": [_vp, _l, _l, _vp, _vp, _i, _vp, _i, _vp, _i, _l, _l, _l,
                         _i, _i, _i, _i, _i, _f, _vp],
    "tllm_gqa_rows": [_vp, _l, _l, _vp, _vp, _i, _vp, _vp, _vp, _i, _l, _l, _l,
                      _i, _i, _i, _i, _i, _i, _i, _f, _vp, _sz, _vp, _vp],
    "tllm_gqa_rows_hint": [_vp, _l, _l, _vp, _vp, _i, _vp, _vp, _vp, _i, _l, _l, _l,
                           _i, _i, _i, _i, _i, _i, _i, _f, _vp, _sz, _vp, _l, _vp],
    # projections
    "tllm_linear_workspace": [_i, _i, _i, _psz, _psz],
    "tllm_linear_plan": [_i, _i, _i, _i, _pi],
    "tllm_linear_fold_parts": [_i, _i, _i, _pi],
    "tllm_linear": [_vp, _i, _i, _vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _i,
                    _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                    _vp, _vp, _vp, _sz, _vp, _vp],
    "tllm_linear_folded": [_vp, _i, _i, _vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _i,
                           _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                           _vp, _vp, _vp, _sz, _vp, _vp, _vp],
    "tllm_gemm_f32": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "tllm_mlp_workspace": [_i, _i, _i, _i, _psz],
    "tllm_mlp": [_vp, _i, _vp, _vp, _vp, _f, _vp, _i, _vp, _vp, _i, _vp, _i, _i, _i, _i,
                 _vp, _sz, _vp],
    # rows / elementwise
    "tllm_rmsnorm": [_vp, _vp, _vp, _i, _i, _i, _i, _f, _vp],
    "tllm_rmsnorm_add": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp],
    "tllm_rmsnorm_p2p": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp],
    # peer group
    "tllm_p2p_handle_bytes": [],
    "tllm_p2p_create": [_i, _i, _i, ctypes.POINTER(_vp), _vp],
    "tllm_p2p_open": [_vp, _i, _vp],
    "tllm_p2p_destroy": [_vp],
    # NCCL (tensor-parallel all-reduce)
    "tllm_nccl_version": [_pi],
    "tllm_nccl_unique_id_bytes": [],
    "tllm_nccl_unique_id": [_vp],
    "tllm_nccl_init": [ctypes.POINTER(ctypes.c_void_p), _i, _i, _vp, _i],
    "tllm_nccl_all_reduce": [_vp, _vp, _sz, _i, _vp, _i],
    "tllm_nccl_check": [_vp, _pi],
    "tllm_nccl_destroy": [_vp, _i],
    "tllm_nccl_abort": [_vp],
    "tllm_layernorm": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp],
    "tllm_split_bf16": [_vp, _vp, _i, _i, _i, _i, _vp],
    "tllm_embedding": [_vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "tllm_argmax": [_vp, _i, _i, _i, _vp, _vp, _vp],
    "tllm_sample": [_vp, _i, _i, _i, _f, _i, _vp, _vp, _vp, _vp],
    "tllm_rope": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "tllm_elementwise": [_i, _vp, _vp, _vp, _l, _vp],
    "tllm_softmax": [_vp, _vp, _i, _i, _vp],
    "tllm_fill_random": [_vp, _i, _l, ctypes.c_uint64, _f, _vp],
}

EPI_STORE, EPI_RESID, EPI_GELU, EPI_SWIGLU, EPI_QKV, EPI_SCATTER = 0, 1, 2, 3, 4, 5


class NormFold(ctypes.Structure):
    """tllm_norm_fold (include/tllm.h): an RMSNorm folded into the
    projections on either side of it."""
    _fields_ = [("next_norm_w", _vp), ("fx", _vp), ("fx_dtype", _i),
                ("fx_plane_rows", _i), ("ss_out", _vp), ("ss_in", _vp),
                ("ss_parts", _i), ("ss_cols", _i), ("eps", _f), ("ss_ld", _i)]
EL_SWIGLU, EL_ADD, EL_GELU = 0, 1, 2

_lib = None
_lock = threading.Lock()


def load():
    """Load libtllm.so once; raises RuntimeError('Failed to load ...')."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = os.environ.get("TLLM_LIB", str(LIB_PATH))
        try:
            lib = ctypes.CDLL(path)
        except OSError as e:
            raise RuntimeError(
                f"Failed to load libtllm.so from {path}: {e}. Build it with "
                "`python triton-llm_b200/csrc/build.py`.") from e
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        lib.tllm_last_error_string.argtypes = []
        lib.tllm_last_error_string.restype = ctypes.c_char_p
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().tllm_last_error_string()
    return msg.decode(errors="replace") if msg else ""


def check(status: int, what: str = "") -> None:
    """Raise the Python exception matching a tllm_status."""
    if status == OK:
        return
    msg = last_error()
    where = f"{what}: " if what else ""
    if status == ERR_INVALID_ARG:
        raise ValueError(f"{where}{msg}")
    if status == ERR_NO_DEVICE:
        raise RuntimeError(
            "No supported GPU runtime found. libtllm.so loaded but no CUDA "
            f"device is visible ({msg}).")
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{where}{msg}")
    raise RuntimeError(f"GPU runtime error (cuda): {status} ({where}{msg})")


def call(name: str, *args) -> None:
    """Call a tllm_* entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def ptr(x) -> int | None:
    """Raw device address of a DeviceTensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()
