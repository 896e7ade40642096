"""Collectives of the tensor-parallel decode (KV-head sharding).

The row-parallel projections (o_proj, down_proj) of a KV-head-sharded model
produce partial sums that every rank needs in full. ``TPGroup.all_reduce``
sums a device buffer across the group with NCCL over NVLink, called from
libtllm.so (``tllm_nccl_all_reduce``) on the library stream like the kernels
around it, so it orders after the projection, before the next kernel, and
can be captured in the decode step's CUDA graph.

``PeerGroup`` is the fused alternative for the decode rows: the projection
epilogue (tllm_linear op SCATTER) writes its partial rows into every rank's
receive slots over NVLink and the next RMSNorm (tllm_rmsnorm_p2p) sums them,
so the all-reduce costs no kernel of its own and no NCCL call.

The host-side plumbing -- the NCCL unique id, the CUDA IPC handles of the
receive slots, barriers -- goes over ``triton_llm.rendezvous`` (TCP, standard
library only), so nothing here needs PyTorch.
"""

from __future__ import annotations

import ctypes

from triton_llm import _lib, gpu
from triton_llm.rendezvous import Rendezvous


class TPGroup:
    """Rank ``rank`` of a tensor-parallel group of ``size`` ranks, one per GPU,
    on CUDA device ``device``. ``rdzv`` is the group's host rendezvous
    (default: ``Rendezvous.from_env()`` when size > 1). ``timeout_ms`` bounds
    every NCCL wait (init, enqueue, destroy)."""

    def __init__(self, rank: int, size: int, device: int,
                 rdzv: Rendezvous | None = None, timeout_ms: int = 120000):
        self.rank, self.size, self.device = int(rank), int(size), int(device)
        self.timeout_ms = int(timeout_ms)
        gpu.set_device(self.device)
        self.rdzv = rdzv
        self._own_rdzv = False
        self.comm = None
        if self.size > 1:
            if self.rdzv is None:
                self.rdzv = Rendezvous.from_env()
                self._own_rdzv = True
            lib = _lib.load()
            uid = ctypes.create_string_buffer(lib.tllm_nccl_unique_id_bytes())
            if self.rank == 0:
                _lib.call("tllm_nccl_unique_id", uid)
            uid_all = self.rdzv.broadcast(uid.raw if self.rank == 0 else None)
            comm = ctypes.c_void_p()
            _lib.call("tllm_nccl_init", ctypes.byref(comm), self.size, self.rank,
                      ctypes.create_string_buffer(uid_all, len(uid_all)),
                      self.timeout_ms)
            self.comm = comm.value

    def all_reduce(self, t):
        """In-place sum of a float32 DeviceTensor over the group, queued on
        the library stream (capturable in a CUDA graph)."""
        if self.size == 1:
            return t
        _lib.call("tllm_nccl_all_reduce", self.comm, t.ptr, int(t.nbytes // 4),
                  _lib.F32, None, self.timeout_ms)
        return t

    def healthy(self) -> bool:
        """False once the communicator reported an error or was aborted."""
        if self.comm is None:
            return True
        st = ctypes.c_int(0)
        _lib.call("tllm_nccl_check", self.comm, ctypes.byref(st))
        return st.value in (0, 7)

    def barrier(self):
        """Wait for this rank's GPU work, then for every rank (host side)."""
        gpu.device_synchronize()
        if self.size > 1:
            self.rdzv.barrier()

    def all_gather_bytes(self, data: bytes) -> list[bytes]:
        if self.size == 1:
            return [bytes(data)]
        return self.rdzv.all_gather(data)

    def peer_group(self, rows: int, cols: int) -> "PeerGroup":
        return PeerGroup(self, rows, cols)

    def close(self):
        """Destroy the communicator (every rank, after its last collective)."""
        if self.comm is not None:
            gpu.device_synchronize()
            comm, self.comm = self.comm, None
            _lib.call("tllm_nccl_destroy", comm, self.timeout_ms)
        if self._own_rdzv and self.rdzv is not None:
            self.rdzv.close()
            self.rdzv = None

    def abort(self):
        """Drop the communicator without waiting for peers (error paths)."""
        if self.comm is not None:
            comm, self.comm = self.comm, None
            _lib.call("tllm_nccl_abort", comm)


class PeerGroup:
    """Receive slots of the fused peer-to-peer all-reduce for up to ``rows``
    rows of ``cols`` fp32 values (tllm_p2p_create / tllm_p2p_open). The CUDA
    IPC handles are exchanged over the group's rendezvous; every rank of
    ``tp`` must construct it, in the same order as its other exchanges."""

    def __init__(self, tp: TPGroup, rows: int, cols: int):
        lib = _lib.load()
        self.rows, self.cols, self.size = int(rows), int(cols), tp.size
        handle = ctypes.create_string_buffer(lib.tllm_p2p_handle_bytes())
        ctx = ctypes.c_void_p()
        _lib.call("tllm_p2p_create", tp.size, self.rows, self.cols, ctypes.byref(ctx),
                  handle)
        self.ctx = ctx.value
        try:
            handles = tp.all_gather_bytes(handle.raw)
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
