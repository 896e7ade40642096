"""Collectives of the tensor-parallel decode (KV-head sharding).

The row-parallel projections (o_proj, down_proj) of a KV-head-sharded model
produce partial sums that every rank needs in full. ``TPGroup.all_reduce``
sums a device buffer across the group with NCCL over NVLink, ordered on the
library stream like the kernels around it (torch's current stream is set to
the library stream, so NCCL waits for the projection and the next kernel
waits for NCCL); it can be captured in the decode step's CUDA graph.
torch.distributed is used only for this plumbing.

``PeerGroup`` is the fused alternative for the decode rows: the projection
epilogue (tllm_linear op SCATTER) writes its partial rows into every rank's
receive slots over NVLink and the next RMSNorm (tllm_rmsnorm_p2p) sums them,
so the all-reduce costs no kernel of its own and no NCCL call.
"""

from __future__ import annotations

import ctypes

from triton_llm import _lib, gpu


class _CudaArray:
    """__cuda_array_interface__ view of a DeviceTensor (no copy)."""

    def __init__(self, t):
        typestr = {4: "<f4", 2: "<u2"}[t.dtype.itemsize] if t.dtype.kind != "i" else "<i4"
        self.__cuda_array_interface__ = {
            "shape": tuple(t.shape), "typestr": typestr,
            "data": (t.data_ptr(), False), "version": 3, "stream": None}


class TPGroup:
    """A tensor-parallel group: rank ``rank`` of ``size`` on CUDA device
    ``device``, NCCL communicator from ``torch.distributed`` (the default
    group if it is NCCL, else a new NCCL group over all ranks)."""

    def __init__(self, rank: int, size: int, device: int):
        import torch
        import torch.distributed as dist
        self.rank, self.size, self.device = rank, size, device
        self._torch, self._dist = torch, dist
        gpu.set_device(device)
        torch.cuda.set_device(device)
        self._stream = torch.cuda.ExternalStream(gpu.stream(), device=device)
        torch.cuda.set_stream(self._stream)
        self.group = None
        if size > 1:
            import datetime
            if dist.get_backend() == "nccl":
                self.group = dist.group.WORLD
            else:
                self.group = dist.new_group(backend="nccl",
                                            timeout=datetime.timedelta(seconds=120))
        self._views = {}

    def _view(self, t):
        key = (t.data_ptr(), tuple(t.shape))
        v = self._views.get(key)
        if v is None:
            v = self._torch.as_tensor(_CudaArray(t), device=f"cuda:{self.device}")
            self._views[key] = v
        return v

    def all_reduce(self, t):
        """In-place sum of a float32 DeviceTensor over the group."""
        if self.size == 1:
            return t
        with self._torch.cuda.stream(self._stream):
            self._dist.all_reduce(self._view(t), group=self.group)
        return t

    def barrier(self):
        if self.size > 1:
            self._dist.barrier(group=self.group, device_ids=[self.device])

    def peer_group(self, rows: int, cols: int) -> "PeerGroup":
        return PeerGroup(self, rows, cols)


class PeerGroup:
    """Receive slots of the fused peer-to-peer all-reduce for up to ``rows``
    rows of ``cols`` fp32 values (tllm_p2p_create / tllm_p2p_open). The CUDA
    IPC handles are exchanged with ``all_gather_object``; every rank of
    ``tp`` must construct it, in the same order as its other collectives."""

    def __init__(self, tp: TPGroup, rows: int, cols: int):
        lib = _lib.load()
        self.rows, self.cols, self.size = int(rows), int(cols), tp.size
        handle = ctypes.create_string_buffer(lib.tllm_p2p_handle_bytes())
        ctx = ctypes.c_void_p()
        _lib.call("tllm_p2p_create", tp.size, self.rows, self.cols, ctypes.byref(ctx),
                  handle)
        self.ctx = ctx.value
        try:
            handles = [handle.raw]
            if tp.size > 1:
                handles = [None] * tp.size
                tp._dist.all_gather_object(handles, handle.raw, group=tp.group)
            _lib.call("tllm_p2p_open", self.ctx, tp.rank, b"".join(handles))
        except Exception:
            self.close()
            raise
        self._tp = tp

    def close(self):
        """Unmap the peers' slots and free this rank's. Call on every rank
        after the last use (a barrier first keeps a peer from still writing)."""
        if self.ctx is not None:
            _lib.call("tllm_p2p_destroy", self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
