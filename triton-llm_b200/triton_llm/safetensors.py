"""Safetensors checkpoints without torch.

The reference converts a HuggingFace checkpoint to one fp32 ``.npy`` file
per tensor through ``safetensors.torch`` (scripts/serve_model.py:155-218,
scripts/download_smollm2_weights.py) and then loads the directory
(scripts/run_smollm2.py:23-48). Here the ``.safetensors`` files are read
directly: the header is parsed, the data section is memory-mapped, and a
tensor is converted to a numpy array only when the model builder asks for
it, so a bf16 checkpoint goes to the device's bf16 weight layout one tensor
at a time (bf16 -> fp32 is exact, and the device rounding back to bf16
returns the same bits) with no fp32 copy of the whole model on the host.

File format (https://github.com/huggingface/safetensors): an 8-byte
little-endian header length N, N bytes of JSON
``{name: {"dtype": "BF16", "shape": [...], "data_offsets": [begin, end]}}``
(plus an optional ``"__metadata__"`` entry), then the data section; offsets
are relative to its start. A sharded checkpoint adds
``model.safetensors.index.json`` with a ``"weight_map"`` of name -> file.
"""

from __future__ import annotations

import json
import mmap
import os
import struct
from collections.abc import Mapping

import numpy as np

_NP = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "I64": np.int64,
       "I32": np.int32, "I16": np.int16, "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_}
_MAX_HEADER = 100 << 20


def _bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


class SafetensorsFile:
    """One ``.safetensors`` file: its header and a read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            raw = f.read(8)
            if len(raw) != 8:
                raise ValueError(f"{path}: not a safetensors file (too short)")
            (n,) = struct.unpack("<Q", raw)
            if n == 0 or n > _MAX_HEADER:
                raise ValueError(f"{path}: header length {n} out of range")
            header = f.read(n)
            if len(header) != n:
                raise ValueError(f"{path}: truncated header")
            try:
                meta = json.loads(header)
            except json.JSONDecodeError as e:
                raise ValueError(f"{path}: header is not JSON ({e})") from None
            size = os.fstat(f.fileno()).st_size
            self._map = (mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
                         if size > 0 else None)
        self.metadata = meta.pop("__metadata__", {})
        self.base = 8 + n
        self.entries = {}
        for name, e in meta.items():
            dt, shape, (b, end) = e["dtype"], tuple(e["shape"]), e["data_offsets"]
            if dt != "BF16" and dt not in _NP:
                raise ValueError(f"{path}: tensor {name} has unsupported dtype {dt}")
            item = 2 if dt == "BF16" else np.dtype(_NP[dt]).itemsize
            if end - b != item * int(np.prod(shape, dtype=np.int64)) or \
                    self.base + end > size or b < 0:
                raise ValueError(f"{path}: tensor {name} has inconsistent offsets")
            self.entries[name] = (dt, shape, b, end)

    def keys(self):
        return self.entries.keys()

    def raw(self, name: str) -> tuple[str, np.ndarray]:
        """(dtype, array view over the file) -- BF16 as uint16 bits."""
        dt, shape, b, end = self.entries[name]
        npdt = np.uint16 if dt == "BF16" else _NP[dt]
        arr = np.frombuffer(self._map, dtype=npdt, count=(end - b) // np.dtype(npdt).itemsize,
                            offset=self.base + b)
        return dt, arr.reshape(shape)

    def get(self, name: str) -> np.ndarray:
        """The tensor as float32 (floating dtypes) or its own integer dtype."""
        dt, arr = self.raw(name)
        if dt == "BF16":
            return _bf16_to_f32(arr)
        if arr.dtype.kind == "f":
            return arr.astype(np.float32)
        return np.array(arr)


class StateDict(Mapping):
    """Name -> numpy array over one file, a list of files, or a checkpoint
    directory (``model.safetensors`` or an index with shards). Arrays are
    made on access; floating tensors come back as float32."""

    def __init__(self, path: str | os.PathLike | list):
        if isinstance(path, (list, tuple)):
            files = [str(p) for p in path]
        elif os.path.isdir(path):
            index = os.path.join(path, "model.safetensors.index.json")
            single = os.path.join(path, "model.safetensors")
            if os.path.exists(index):
                with open(index) as f:
                    wm = json.load(f)["weight_map"]
                files = [os.path.join(path, s) for s in sorted(set(wm.values()))]
            elif os.path.exists(single):
                files = [single]
            else:
                files = sorted(os.path.join(path, p) for p in os.listdir(path)
                               if p.endswith(".safetensors"))
            if not files:
                raise FileNotFoundError(f"no .safetensors files in {path}")
        else:
            files = [str(path)]
        self.files = [SafetensorsFile(p) for p in files]
        self._where = {}
        for f in self.files:
            for k in f.keys():
                if k in self._where:
                    raise ValueError(f"tensor {k} appears in two files")
                self._where[k] = f

    def __getitem__(self, name):
        return self._where[name].get(name)

    def raw(self, name):
        return self._where[name].raw(name)

    def __iter__(self):
        return iter(self._where)

    def __len__(self):
        return len(self._where)


def load_state_dict(path) -> StateDict:
    """A lazily converted state dict of a safetensors checkpoint."""
    return StateDict(path)


def save_file(tensors: dict, path: str, bf16: bool = False, metadata: dict | None = None):
    """Write ``tensors`` (name -> numpy array) as one ``.safetensors`` file;
    floating arrays are stored as BF16 (round to nearest even) when
    ``bf16`` is set, else as F32."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        if a.dtype.kind == "f":
            if bf16:
                u = np.ascontiguousarray(a, np.float32).view(np.uint32)
                bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
                nan = np.isnan(np.ascontiguousarray(a, np.float32))
                bits[nan] = 0x7FC0
                data, dt = bits.tobytes(), "BF16"
            else:
                data, dt = np.ascontiguousarray(a, np.float32).tobytes(), "F32"
        else:
            rev = {v: k for k, v in _NP.items()}
            if a.dtype.type not in rev:
                raise ValueError(f"{name}: unsupported dtype {a.dtype}")
            data, dt = a.tobytes(), rev[a.dtype.type]
        header[name] = {"dtype": dt, "shape": list(a.shape),
                        "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)   # align the data section
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
