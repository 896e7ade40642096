"""Host-side meeting point of the ranks of one node, over TCP.

The tensor-parallel decode needs a few host-side exchanges before its data
plane runs on the GPUs: the NCCL unique id made by rank 0, every rank's CUDA
IPC handle of its peer-all-reduce receive slots, and barriers around set-up,
timed regions and tear-down. ``Rendezvous`` provides exactly that --
``all_gather`` of small byte strings and ``barrier`` -- with the standard
library only (no torch.distributed): rank 0 serves a socket, every rank
(rank 0 included) connects to it, and each operation is one round in which
the server collects one message per rank, in rank order, and sends the
concatenation back to all of them.

Failures end in an exception, never a hang: every blocking step has a
deadline (``timeout``), a rank that leaves (its socket closes) makes the
server close every connection, and the other ranks' current or next
operation raises ``RuntimeError``; a rank that never arrives makes the
others' operation raise ``TimeoutError``.

Ranks find the server at ``addr:port``; ``from_env`` reads RANK,
WORLD_SIZE and MASTER_ADDR from the environment (as torchrun sets them) and
uses port ``TLLM_RDZV_PORT``, or ``MASTER_PORT + 1`` (torchrun's own store
holds MASTER_PORT).
"""

from __future__ import annotations

import os
import socket
import struct
import threading
import time

_MAGIC = 0x544C4C4D          # "TLLM"
_HDR = struct.Struct("!IiI")  # magic, rank, world
_LEN = struct.Struct("!q")    # payload length (-1: the group failed)


def _recv_exact(sock: socket.socket, n: int, deadline: float) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        left = deadline - time.monotonic()
        if left <= 0:
            raise TimeoutError
        sock.settimeout(min(left, 1.0))
        try:
            chunk = sock.recv(n - len(buf))
        except socket.timeout:
            continue
        if not chunk:
            raise ConnectionError("connection closed")
        buf += chunk
    return bytes(buf)


class _Server(threading.Thread):
    """Rank 0's server: accepts ``world`` connections, then runs rounds."""

    def __init__(self, addr: str, port: int, world: int, timeout: float):
        super().__init__(daemon=True, name="tllm-rendezvous")
        self.world, self.timeout = world, timeout
        self.lsock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.lsock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.lsock.bind((addr, port))
        self.lsock.listen(world)
        self.port = self.lsock.getsockname()[1]
        self.conns: list[socket.socket | None] = [None] * world
        self.error: str | None = None
        self._halt = threading.Event()

    def run(self):
        try:
            self._accept()
            while not self._halt.is_set():
                msgs = []
                for r in range(self.world):
                    msgs.append(self._read(r))
                out = b"".join(_LEN.pack(len(m)) + m for m in msgs)
                for c in self.conns:
                    c.sendall(out)
        except Exception as e:  # a rank left, timed out, or the group closed
            if not self._halt.is_set():
                self.error = f"{type(e).__name__}: {e}"
        finally:
            self._close_all()

    def _accept(self):
        deadline = time.monotonic() + self.timeout
        n = 0
        while n < self.world:
            left = deadline - time.monotonic()
            if left <= 0:
                missing = [r for r, c in enumerate(self.conns) if c is None]
                raise TimeoutError(f"ranks {missing} never connected")
            self.lsock.settimeout(min(left, 1.0))
            try:
                c, _ = self.lsock.accept()
            except socket.timeout:
                continue
            c.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            magic, rank, world = _HDR.unpack(_recv_exact(c, _HDR.size, deadline))
            if magic != _MAGIC or world != self.world or not 0 <= rank < world \
                    or self.conns[rank] is not None:
                c.close()
                continue
            self.conns[rank] = c
            n += 1

    def _read(self, r: int) -> bytes:
        # an idle group may wait between operations for as long as it likes;
        # a closed connection ends it at once
        c = self.conns[r]
        (n,) = _LEN.unpack(_recv_exact(c, _LEN.size, float("inf")))
        if n < 0:
            raise ConnectionError(f"rank {r} closed the group")
        return _recv_exact(c, n, time.monotonic() + self.timeout)

    def _close_all(self):
        for c in self.conns:
            if c is not None:
                try:
                    c.sendall(_LEN.pack(-1))
                except OSError:
                    pass
                try:
                    c.close()
                except OSError:
                    pass
        try:
            self.lsock.close()
        except OSError:
            pass

    def stop(self):
        self._halt.set()


class Rendezvous:
    """Rank ``rank`` of ``world`` ranks meeting at ``addr:port``."""

    def __init__(self, rank: int, world: int, addr: str = "127.0.0.1",
                 port: int = 0, timeout: float = 120.0):
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} of {world} is invalid")
        self.rank, self.world, self.timeout = int(rank), int(world), float(timeout)
        self.server = None
        self.sock = None
        self._rounds = 0
        if world == 1:
            return
        if rank == 0:
            self.server = _Server(addr, port, world, timeout)
            self.server.start()
            port = self.server.port
        self.addr, self.port = addr, port
        self._connect(addr, port)

    @classmethod
    def from_env(cls, timeout: float = 120.0) -> "Rendezvous":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = os.environ.get("TLLM_RDZV_PORT")
        if port is None:
            port = int(os.environ.get("MASTER_PORT", "29500")) + 1
        return cls(rank, world, addr, int(port), timeout)

    def _connect(self, addr, port):
        deadline = time.monotonic() + self.timeout
        while True:
            try:
                s = socket.create_connection((addr, port), timeout=1.0)
                break
            except OSError:
                if time.monotonic() > deadline:
                    raise TimeoutError(f"rank {self.rank}: no rendezvous server at "
                                       f"{addr}:{port} after {self.timeout:.0f} s")
                time.sleep(0.05)
        s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        s.sendall(_HDR.pack(_MAGIC, self.rank, self.world))
        self.sock = s

    def all_gather(self, data: bytes, timeout: float | None = None) -> list[bytes]:
        """Every rank's ``data``, in rank order (the same list on every rank)."""
        data = bytes(data)
        if self.world == 1:
            return [data]
        if self.sock is None:
            raise RuntimeError("rendezvous is closed")
        timeout = self.timeout if timeout is None else float(timeout)
        deadline = time.monotonic() + timeout
        self._rounds += 1
        try:
            self.sock.sendall(_LEN.pack(len(data)) + data)
            out = []
            for r in range(self.world):
                (n,) = _LEN.unpack(_recv_exact(self.sock, _LEN.size, deadline))
                if n < 0:
                    raise ConnectionError("the group was closed")
                out.append(_recv_exact(self.sock, n, deadline))
            return out
        except TimeoutError:
            self._fail()
            raise TimeoutError(
                f"rank {self.rank}: rendezvous round {self._rounds} timed out after "
                f"{timeout:.1f} s (a rank did not arrive)") from None
        except (ConnectionError, OSError) as e:
            why = self.server.error if self.server is not None else None
            self._fail()
            raise RuntimeError(
                f"rank {self.rank}: rendezvous round {self._rounds} failed: a rank "
                f"left the group ({why or e})") from None

    def barrier(self, timeout: float | None = None) -> None:
        self.all_gather(b"", timeout)

    def broadcast(self, data: bytes | None, root: int = 0,
                  timeout: float | None = None) -> bytes:
        return self.all_gather(data if self.rank == root else b"", timeout)[root]

    def reduce_max(self, x: float) -> float:
        return max(float(v) for v in self.all_gather(repr(float(x)).encode()))

    def reduce_sum(self, x: float) -> float:
        return sum(float(v) for v in self.all_gather(repr(float(x)).encode()))

    def _fail(self):
        if self.sock is not None:
            try:
                self.sock.close()
            except OSError:
                pass
            self.sock = None
        if self.server is not None:
            self.server.stop()
            self.server._close_all()

    def close(self) -> None:
        """Leave the group (after the last operation every rank takes part in)."""
        if self.sock is not None:
            try:
                self.sock.sendall(_LEN.pack(-1))
            except OSError:
                pass
        if self.server is not None:
            self.server.stop()
            self.server.join(timeout=5)
        self._fail()

    def __del__(self):
        try:
            self._fail()
        except Exception:
            pass
