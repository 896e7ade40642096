"""The host rendezvous of the multi-GPU paths (triton_llm.rendezvous) and
the NCCL binding's host side, on CPU.

Ranks are spawned processes on 127.0.0.1. Failures are made on the host: a
rank that never arrives at an operation, a rank that leaves the group, a
rank that never connects; each must end the other ranks' waits with an
exception within the timeout, never a hang.
"""

from __future__ import annotations

import ctypes
import multiprocessing as mp
import os
import socket
import subprocess
import sys
import time
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, mode, q):
    sys.path.insert(0, str(REPO / "triton-llm_b200"))
    from triton_llm.rendezvous import Rendezvous
    try:
        r = Rendezvous(rank, world, "127.0.0.1", port, timeout=3.0)
        if mode == "ok":
            got = r.all_gather(f"rank{rank}".encode() * (rank + 1))
            r.barrier()
            b = r.broadcast(b"id-from-0" if rank == 0 else None)
            mx = r.reduce_max(float(rank * 10))
            sm = r.reduce_sum(1.5)
            for i in range(20):            # many small rounds in a row
                assert r.all_gather(bytes([i, rank]))[world - 1] == bytes([i, world - 1])
            r.close()
            q.put((rank, "ok", [g.decode() for g in got], b.decode(), mx, sm))
        elif mode == "straggler":
            if rank == world - 1:
                time.sleep(6.0)            # never arrives within the timeout
                r.close()
                q.put((rank, "slept"))
                return
            t = time.monotonic()
            try:
                r.all_gather(b"x", timeout=1.5)
                q.put((rank, "no error"))
            except (TimeoutError, RuntimeError) as e:
                q.put((rank, type(e).__name__, time.monotonic() - t))
        elif mode == "leaver":
            if rank == world - 1:
                r.close()                  # leaves before the first round
                q.put((rank, "left"))
                return
            t = time.monotonic()
            try:
                r.all_gather(b"x", timeout=5.0)
                q.put((rank, "no error"))
            except (TimeoutError, RuntimeError) as e:
                q.put((rank, type(e).__name__, time.monotonic() - t))
    except Exception as e:  # pragma: no cover - reported to the test
        q.put((rank, "exception", repr(e)))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q))
          for r in range(world)]
    for p in ps:
        p.start()
    out = sorted((q.get(timeout=60) for _ in range(world)), key=lambda x: x[0])
    for p in ps:
        p.join(timeout=30)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("world", [2, 4])
def test_rendezvous_collectives(world):
    out = _run(world, "ok")
    want = [f"rank{r}" * (r + 1) for r in range(world)]
    for rank, status, got, b, mx, sm in out:
        assert status == "ok"
        assert got == want
        assert b == "id-from-0"
        assert mx == 10.0 * (world - 1)
        assert sm == pytest.approx(1.5 * world)


def test_rendezvous_rank_that_never_arrives_times_out():
    out = _run(3, "straggler")
    for rank, status, *rest in out[:2]:
        assert status in ("TimeoutError", "RuntimeError"), (rank, status, rest)
        assert rest[0] < 4.0               # bounded by the 1.5 s limit (+ slack)
    assert out[2][1] == "slept"


def test_rendezvous_rank_that_leaves_fails_the_others():
    out = _run(3, "leaver")
    for rank, status, *rest in out[:2]:
        assert status == "RuntimeError", (rank, status, rest)
        assert rest[0] < 4.0
    assert out[2][1] == "left"


def test_rendezvous_rank_that_never_connects():
    sys.path.insert(0, str(REPO / "triton-llm_b200"))
    from triton_llm.rendezvous import Rendezvous
    t = time.monotonic()
    r = Rendezvous(0, 2, "127.0.0.1", _port(), timeout=1.0)
    with pytest.raises((TimeoutError, RuntimeError)):
        r.all_gather(b"x")
    assert time.monotonic() - t < 5.0
    r.close()


def test_rendezvous_single_rank_needs_no_server():
    sys.path.insert(0, str(REPO / "triton-llm_b200"))
    from triton_llm.rendezvous import Rendezvous
    r = Rendezvous(0, 1)
    assert r.all_gather(b"a") == [b"a"]
    r.barrier()
    assert r.reduce_max(3.0) == 3.0
    r.close()


# ---------------------------------------------------------- NCCL binding ----
def test_nccl_loads_and_makes_unique_ids():
    """libtllm.so binds NCCL by dlopen; the version query and the unique id
    need no GPU."""
    from triton_llm import _lib
    lib = _lib.load()
    v = ctypes.c_int(0)
    _lib.call("tllm_nccl_version", ctypes.byref(v))
    assert v.value >= 21900
    n = lib.tllm_nccl_unique_id_bytes()
    assert n == 128
    a, b = ctypes.create_string_buffer(n), ctypes.create_string_buffer(n)
    _lib.call("tllm_nccl_unique_id", a)
    _lib.call("tllm_nccl_unique_id", b)
    assert a.raw != b.raw and any(a.raw)


def test_nccl_argument_checks_and_missing_library():
    from triton_llm import _lib
    lib = _lib.load()
    comm = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(128)
    assert lib.tllm_nccl_init(ctypes.byref(comm), 2, 2, uid, 100) == _lib.ERR_INVALID_ARG
    assert lib.tllm_nccl_all_reduce(None, None, 4, _lib.F32, None, 100) == _lib.ERR_INVALID_ARG
    assert lib.tllm_nccl_destroy(None, 100) == _lib.OK
    # a process whose NCCL library cannot be found reports TLLM_ERR_NCCL
    code = (
        "import sys, ctypes; sys.path.insert(0, 'triton-llm_b200');"
        "from triton_llm import _lib; lib = _lib.load(); v = ctypes.c_int();"
        "st = lib.tllm_nccl_version(ctypes.byref(v));"
        "print(st, _lib.last_error())")
    env = dict(os.environ, TLLM_NCCL_LIB="/nonexistent/libnccl.so.2")
    r = subprocess.run([sys.executable, "-c", code], cwd=str(REPO), env=env,
                       capture_output=True, text=True, timeout=60)
    st, msg = r.stdout.split(" ", 1)
    assert int(st) == _lib.ERR_NCCL and "NCCL library unavailable" in msg


def test_nccl_fault_injection():
    code = (
        "import sys, ctypes; sys.path.insert(0, 'triton-llm_b200');"
        "from triton_llm import _lib; lib = _lib.load();"
        "b = ctypes.create_string_buffer(128);"
        "print(lib.tllm_nccl_unique_id(b), lib.tllm_nccl_unique_id(b))")
    env = dict(os.environ, TLLM_FAULT_INJECT="nccl:2")
    r = subprocess.run([sys.executable, "-c", code], cwd=str(REPO), env=env,
                       capture_output=True, text=True, timeout=60)
    from triton_llm import _lib
    assert r.stdout.split() == ["0", str(_lib.ERR_INJECTED)], r.stdout + r.stderr
