"""Run the reference triton-llm on the CPU (TRITON_INTERPRET=1).

Test infrastructure only: used by ``gen_golden.py`` in the development
container where the reference checkout is readable. Nothing in the product,
``bench.py`` or the GPU tests imports this module.

The reference's kernels take raw device addresses from
``triton_llm.gpu.DeviceTensor.data_ptr()``. Under the Triton interpreter those
addresses are dereferenced as host memory, so the GPU allocator is replaced by
a host stand-in with the same API whose buffers are anonymous ``mmap`` regions
(their addresses are above 2**31, which the interpreter needs to type the
integer arguments as 64-bit pointers).
"""

from __future__ import annotations

import ctypes
import mmap
import os
import sys

import numpy as np



class HostTensor:
    """Host-memory DeviceTensor (same attributes as triton_llm/gpu.py:184-227)."""

    def __init__(self, shape, dtype, nbytes, buf=None, defer_free=True):
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)
        self.nbytes = int(nbytes)
        self._defer_free = defer_free
        if buf is None:
            buf = mmap.mmap(-1, max(self.nbytes, 1))
        self._buf = buf
        arr = np.frombuffer(buf, dtype=np.uint8)
        self._addr = arr.ctypes.data
        self.ptr = ctypes.c_void_p(self._addr)

    def _array(self):
        return np.frombuffer(self._buf, dtype=self.dtype,
                             count=int(np.prod(self.shape))).reshape(self.shape)

    def to_numpy(self):
        return self._array().copy()

    def from_numpy(self, arr):
        a = np.ascontiguousarray(arr, dtype=self.dtype).reshape(self.shape)
        self._array()[...] = a

    def data_ptr(self):
        return self._addr


def _allocate(shape, dtype=np.float32):
    nbytes = int(np.prod(shape) * np.dtype(dtype).itemsize)
    return HostTensor(shape, dtype, nbytes)


def _to_device(arr):
    t = _allocate(arr.shape, arr.dtype)
    t.from_numpy(arr)
    return t


def _to_host(t):
    return t.to_numpy()


def _synchronize():
    return None


def _view(t, new_shape):
    n_old, n_new = int(np.prod(t.shape)), int(np.prod(new_shape))
    if n_old != n_new:
        raise ValueError(f"Cannot view {t.shape} as {new_shape}")
    v = HostTensor(new_shape, t.dtype, t.nbytes, buf=t._buf, defer_free=False)
    return v


def install(ref_root: str | None = None):
    """Import the reference with the host allocator patched in.

    Returns the reference's ``triton_llm.gpu`` module.
    """
    ref_root = ref_root or os.environ.get("TLLM_REFERENCE")
    if not ref_root:
        raise RuntimeError("set TLLM_REFERENCE to the reference triton-llm checkout")
    os.environ["TRITON_INTERPRET"] = "1"
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    for name in list(sys.modules):
        if name.split(".")[0] in ("triton_llm", "smollm2_triton", "gpt2_triton"):
            mod = sys.modules[name]
            f = getattr(mod, "__file__", "") or ""
            if not f.startswith(ref_root):
                raise RuntimeError(
                    f"{name} already imported from {f}; run the golden generator "
                    "in a process that has not imported the product package")
    import triton_llm.gpu as g  # noqa: E402  (the reference module)
    g.DeviceTensor = HostTensor
    g.allocate = _allocate
    g.to_device = _to_device
    g.to_host = _to_host
    g.synchronize = _synchronize
    g.view = _view
    g._initialize = lambda: None
    return g
