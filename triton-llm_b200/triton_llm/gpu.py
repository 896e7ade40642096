"""GPU memory allocator and device runtime (drop-in for triton_llm/gpu.py).

Same public surface as the reference module (triton_llm/gpu.py:179-294):
``allocate``, ``to_device``, ``to_host``, ``synchronize``, ``view``,
``check_error`` and ``DeviceTensor`` with ``ptr`` / ``shape`` / ``dtype`` /
``nbytes`` / ``data_ptr()`` / ``to_numpy()`` / ``from_numpy()``.

Differences in mechanism, not in contract:

* memory comes from libtllm.so's stream-ordered pool (``cudaMallocAsync``
  on the device's library stream) instead of ``cudaMalloc``; freeing a
  tensor never synchronises the device;
* copies and kernels are ordered on that one stream, and ``synchronize()``
  waits for it;
* the only backend is CUDA on sm_100a (the reference also probes HIP);
* tensors may hold bf16 data: ``allocate(shape, "bfloat16")`` creates a
  tensor whose host representation is ``np.uint16`` bit patterns
  (``DeviceTensor.is_bf16`` is True); ``to_device_bf16`` rounds an fp32
  array to bf16 (round to nearest even) on upload.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

CUDA_MEMCPY_HOST_TO_DEVICE = 1
CUDA_MEMCPY_DEVICE_TO_HOST = 2
CUDA_SUCCESS = 0

BFLOAT16 = "bfloat16"

_initialized = False
_backend = None


def _initialize():
    """Load libtllm.so and check that a CUDA device is visible."""
    global _initialized, _backend
    if _initialized:
        return
    lib = _lib.load()
    n = ctypes.c_int(0)
    _lib.check(lib.tllm_device_count(ctypes.byref(n)), "device_count")
    _backend = "cuda"
    _initialized = True


def check_error(err):
    """Raise on a non-zero status (triton_llm/gpu.py:179-181)."""
    if err != CUDA_SUCCESS:
        raise RuntimeError(f"GPU runtime error ({_backend or 'cuda'}): {err}")


def device_count() -> int:
    lib = _lib.load()
    n = ctypes.c_int(0)
    status = lib.tllm_device_count(ctypes.byref(n))
    return n.value if status == 0 else 0


def set_device(device: int) -> None:
    _initialize()
    _lib.call("tllm_set_device", int(device))


def current_device() -> int:
    _initialize()
    d = ctypes.c_int(0)
    _lib.call("tllm_get_device", ctypes.byref(d))
    return d.value


def _np_dtype(dtype):
    if isinstance(dtype, str) and dtype in ("bfloat16", "bf16"):
        return np.dtype(np.uint16), True
    return np.dtype(dtype), False


class DeviceTensor:
    """Wrapper for a GPU device pointer with automatic cleanup.

    ``ptr`` is a ``ctypes.c_void_p`` exactly as in the reference; a tensor
    created by ``allocate`` owns its memory and releases it in ``__del__``,
    a ``view`` does not (``defer_free=False``) but keeps its base alive.
    """

    def __init__(self, ptr, shape, dtype, nbytes, defer_free=True,
                 is_bf16=False, base=None, device=None):
        self.ptr = ptr
        self.shape = tuple(int(s) for s in shape)
        self.dtype = np.dtype(dtype)
        self.nbytes = int(nbytes)
        self.is_bf16 = bool(is_bf16)
        self._defer_free = defer_free
        self._base = base
        self.device = device
        self.is_split = False   # TLLM_SPLIT activation buffer (split_empty)

    def __del__(self):
        if not getattr(self, "_defer_free", False):
            return
        p = self.ptr.value if self.ptr is not None else None
        if not p or _lib._lib is None:
            return
        try:
            lib = _lib._lib
            cur = ctypes.c_int(0)
            lib.tllm_get_device(ctypes.byref(cur))
            if self.device is not None and cur.value != self.device:
                lib.tllm_set_device(self.device)
                lib.tllm_free(ctypes.c_void_p(p))
                lib.tllm_set_device(cur.value)
            else:
                lib.tllm_free(ctypes.c_void_p(p))
        except Exception:
            pass

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def to_numpy(self):
        _initialize()
        host = np.empty(self.shape, dtype=self.dtype)
        if self.nbytes:
            _lib.check(_lib.load().tllm_memcpy_d2h(
                host.ctypes.data_as(ctypes.c_void_p), self.ptr, self.nbytes),
                "to_numpy")
        return host

    def from_numpy(self, arr: np.ndarray):
        _initialize()
        arr = np.ascontiguousarray(arr)
        if arr.nbytes != self.nbytes:
            raise ValueError(
                f"from_numpy: {arr.nbytes} bytes into a {self.nbytes}-byte tensor")
        if self.nbytes:
            _lib.check(_lib.load().tllm_memcpy_h2d(
                self.ptr, arr.ctypes.data_as(ctypes.c_void_p), self.nbytes),
                "from_numpy")

    def data_ptr(self):
        return self.ptr.value

    def __repr__(self):
        kind = "bfloat16" if self.is_bf16 else str(self.dtype)
        return f"DeviceTensor(shape={self.shape}, dtype={kind}, ptr=0x{self.data_ptr() or 0:x})"


def allocate(shape, dtype=np.float32):
    """Allocate memory on the current GPU (uninitialised, like cudaMalloc)."""
    _initialize()
    if isinstance(shape, int):
        shape = (shape,)
    npd, bf16 = _np_dtype(dtype)
    nbytes = int(np.prod(shape) * npd.itemsize) if len(shape) else npd.itemsize
    ptr = ctypes.c_void_p()
    _lib.check(_lib.load().tllm_malloc(ctypes.byref(ptr), nbytes), "allocate")
    return DeviceTensor(ptr, shape, npd, nbytes, is_bf16=bf16,
                        device=current_device())


def zeros(shape, dtype=np.float32):
    """Allocate and zero-fill (stream ordered)."""
    t = allocate(shape, dtype)
    memset(t, 0)
    return t


def memset(t: DeviceTensor, value: int = 0):
    _lib.call("tllm_memset", t.ptr, int(value), t.nbytes, None)


def to_device(arr: np.ndarray):
    """Copy a numpy array to the GPU."""
    _initialize()
    arr = np.ascontiguousarray(arr)
    tensor = allocate(arr.shape, arr.dtype)
    tensor.from_numpy(arr)
    return tensor


def f32_to_bf16_bits(arr: np.ndarray) -> np.ndarray:
    """Round fp32 -> bf16 (nearest even) and return the uint16 bit patterns."""
    a = np.ascontiguousarray(arr, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded[nan] = ((a.view(np.uint32)[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32)
            << 16).view(np.float32)


def to_device_bf16(arr: np.ndarray):
    """Upload an fp32 array as bf16 (round to nearest even)."""
    bits = f32_to_bf16_bits(arr)
    t = allocate(bits.shape, BFLOAT16)
    t.from_numpy(bits)
    return t


def to_host(tensor: DeviceTensor):
    """Copy a DeviceTensor back to numpy (bf16 tensors come back as fp32)."""
    out = tensor.to_numpy()
    if tensor.is_bf16:
        return bf16_bits_to_f32(out)
    return out


def act_empty(rows: int, cols: int, planes: int = 1) -> DeviceTensor:
    """An activation buffer in a tensor-core operand format: shape
    (planes, rows, cols) of bf16 with plane 0 = bf16(x) and, for planes=2
    (TLLM_SPLIT), plane 1 = bf16(x - hi); planes=1 is TLLM_BF16. Kernels
    that take activations accept it wherever they accept fp32."""
    if planes not in (1, 2):
        raise ValueError(f"planes must be 1 or 2, got {planes}")
    t = allocate((int(planes), int(rows), int(cols)), BFLOAT16)
    t.is_split = True
    return t


def split_empty(rows: int, cols: int) -> DeviceTensor:
    """TLLM_SPLIT activation buffer (hi and lo planes)."""
    return act_empty(rows, cols, 2)


def split_host(arr: np.ndarray):
    """(hi, lo) bf16 bit planes of an fp32 array, as the device computes them."""
    a = np.ascontiguousarray(arr, dtype=np.float32)
    hi = f32_to_bf16_bits(a)
    lo = f32_to_bf16_bits(a - bf16_bits_to_f32(hi))
    return hi, lo


def to_device_split(arr: np.ndarray, plane_rows: int | None = None,
                    planes: int = 2) -> DeviceTensor:
    """Upload an fp32 (rows, cols) array in an operand format (TLLM_SPLIT
    for planes=2, TLLM_BF16 for planes=1)."""
    a = np.ascontiguousarray(arr, dtype=np.float32)
    rows, cols = a.shape
    pr = rows if plane_rows is None else int(plane_rows)
    hi, lo = split_host(a)
    buf = np.zeros((planes, pr, cols), np.uint16)
    buf[0, :rows] = hi
    if planes == 2:
        buf[1, :rows] = lo
    t = act_empty(pr, cols, planes)
    t.from_numpy(buf)
    return t


def split_to_host(t: DeviceTensor, rows: int | None = None) -> np.ndarray:
    """The fp32 values (hi + lo, or hi) of an operand-format buffer."""
    planes = t.to_numpy()
    n = planes.shape[1] if rows is None else int(rows)
    out = bf16_bits_to_f32(planes[0, :n])
    if planes.shape[0] == 2:
        out = out + bf16_bits_to_f32(planes[1, :n])
    return out.astype(np.float32)


def act_args(t: DeviceTensor):
    """(pointer, dtype code, rows per plane) of an activation buffer: fp32
    (rows, cols), TLLM_SPLIT (2, rows, cols) or TLLM_BF16 (1, rows, cols)."""
    if getattr(t, "is_split", False):
        return t.ptr, (_lib.SPLIT if t.shape[0] == 2 else _lib.BF16), int(t.shape[1])
    return t.ptr, _lib.F32, int(t.shape[0])


def synchronize():
    """Wait for all work queued on the library stream of this device."""
    _initialize()
    _lib.call("tllm_synchronize")


def view(tensor: DeviceTensor, new_shape: tuple) -> DeviceTensor:
    """Zero-copy view with a new shape (triton_llm/gpu.py:266-294).

    Raises ``ValueError`` on an element-count mismatch, like the reference.
    """
    n_elems = int(np.prod(tensor.shape))
    n_new = int(np.prod(new_shape))
    if n_elems != n_new:
        raise ValueError(
            f"Cannot view {tensor.shape} ({n_elems} elements) as "
            f"{new_shape} ({n_new} elements) — element count mismatch"
        )
    return DeviceTensor(tensor.ptr, new_shape, tensor.dtype, tensor.nbytes,
                        defer_free=False, is_bf16=tensor.is_bf16,
                        base=tensor, device=tensor.device)


def sub_view(tensor: DeviceTensor, byte_offset: int, shape, dtype=None,
             is_bf16=None) -> DeviceTensor:
    """View of a byte range of ``tensor`` (for slices of one arena)."""
    dtype = tensor.dtype if dtype is None else np.dtype(dtype)
    is_bf16 = tensor.is_bf16 if is_bf16 is None else is_bf16
    nbytes = int(np.prod(shape)) * dtype.itemsize
    if byte_offset < 0 or byte_offset + nbytes > tensor.nbytes:
        raise ValueError("sub_view out of range")
    return DeviceTensor(ctypes.c_void_p(tensor.data_ptr() + byte_offset), shape,
                        dtype, nbytes, defer_free=False, is_bf16=is_bf16,
                        base=tensor, device=tensor.device)


def device_error(reset: bool = True) -> int:
    """Read (and by default clear) the device-side error word."""
    _initialize()
    code = ctypes.c_int(0)
    _lib.call("tllm_device_error", ctypes.byref(code), 1 if reset else 0)
    return code.value


def stream():
    """The library stream handle (an int) of the current device."""
    _initialize()
    s = ctypes.c_void_p()
    _lib.call("tllm_get_stream", ctypes.byref(s))
    return s.value


class Event:
    """CUDA event on the library stream, for device-side timing."""

    def __init__(self):
        _initialize()
        self._e = ctypes.c_void_p()
        _lib.call("tllm_event_create", ctypes.byref(self._e))

    def record(self, stream=None):
        _lib.call("tllm_event_record", self._e, stream)

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0)
        _lib.call("tllm_event_elapsed_ms", self._e, end._e, ctypes.byref(ms))
        return ms.value

    def __del__(self):
        try:
            if _lib._lib is not None and self._e:
                _lib._lib.tllm_event_destroy(self._e)
        except Exception:
            pass


# ---------------------------------------------------------------------------
# Page-locked host buffers and asynchronous copies (end-to-end paths)
# ---------------------------------------------------------------------------
class _PinnedBuffer:
    def __init__(self, nbytes):
        _initialize()
        self.ptr = ctypes.c_void_p()
        _lib.call("tllm_host_alloc", ctypes.byref(self.ptr), max(int(nbytes), 1))
        self.nbytes = int(nbytes)
        self.raw = (ctypes.c_char * max(self.nbytes, 1)).from_address(self.ptr.value)

    def __del__(self):
        try:
            if _lib._lib is not None and self.ptr:
                _lib._lib.tllm_host_free(self.ptr)
        except Exception:
            pass


class PinnedArray(np.ndarray):
    """ndarray over page-locked host memory; the memory lives as long as the
    array (and every view of it) does."""
    _pinned = None

    def __array_finalize__(self, obj):
        if obj is not None:
            self._pinned = getattr(obj, "_pinned", None)


def pinned_empty(shape, dtype=np.float32) -> np.ndarray:
    """numpy array in page-locked host memory (freed with the array)."""
    if isinstance(shape, int):
        shape = (shape,)
    dtype = np.dtype(dtype)
    count = int(np.prod(shape))
    buf = _PinnedBuffer(count * dtype.itemsize)
    arr = np.frombuffer(buf.raw, dtype=dtype, count=count).reshape(shape)
    arr = arr.view(PinnedArray)
    arr._pinned = buf
    return arr


def copy_h2d_async(dst: DeviceTensor, src: np.ndarray, stream=None, nbytes=None):
    n = dst.nbytes if nbytes is None else int(nbytes)
    if n > dst.nbytes or n > src.nbytes or not src.flags["C_CONTIGUOUS"]:
        raise ValueError(f"copy of {n} bytes: device buffer {dst.nbytes}, "
                         f"host buffer {src.nbytes} (contiguous required)")
    _lib.call("tllm_memcpy_h2d_async", dst.ptr,
              src.ctypes.data_as(ctypes.c_void_p), n, stream)


def copy_d2h_async(dst: np.ndarray, src: DeviceTensor, stream=None, nbytes=None):
    n = src.nbytes if nbytes is None else int(nbytes)
    if n > dst.nbytes or n > src.nbytes or not dst.flags["C_CONTIGUOUS"]:
        raise ValueError(f"copy of {n} bytes: device buffer {src.nbytes}, "
                         f"host buffer {dst.nbytes} (contiguous required)")
    _lib.call("tllm_memcpy_d2h_async", dst.ctypes.data_as(ctypes.c_void_p),
              src.ptr, n, stream)


def copy_d2d(dst: DeviceTensor, src: DeviceTensor, nbytes=None):
    n = min(dst.nbytes, src.nbytes) if nbytes is None else int(nbytes)
    _lib.call("tllm_memcpy_d2d", dst.ptr, src.ptr, n)


def stream_synchronize(stream=None):
    _lib.call("tllm_stream_synchronize", stream)


def device_synchronize():
    _lib.call("tllm_device_synchronize")


def mem_info():
    f, t = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.call("tllm_mem_info", ctypes.byref(f), ctypes.byref(t))
    return f.value, t.value


class Graph:
    """A CUDA graph of library work captured on the library stream.

        with gpu.Graph() as g:      # calls inside are recorded, not run
            step()
        g.launch()                  # replays them with one launch
    """

    def __init__(self):
        _initialize()
        self._exec = None

    def __enter__(self):
        _lib.call("tllm_graph_capture_begin", None)
        return self

    def __exit__(self, exc_type, exc, tb):
        e = ctypes.c_void_p()
        status = _lib.load().tllm_graph_capture_end(None, ctypes.byref(e))
        if exc_type is None:
            _lib.check(status, "tllm_graph_capture_end")
            self._exec = e
        return False

    def launch(self):
        _lib.call("tllm_graph_launch", self._exec, None)

    def __del__(self):
        try:
            if _lib._lib is not None and self._exec:
                _lib._lib.tllm_graph_destroy(self._exec)
        except Exception:
            pass
