"""The C ABI library: loads, exports every declared symbol, maps errors.

CPU-only: no kernel is launched. Entry points that need a device are only
called where the call fails before touching the GPU (argument checks and
injected faults), or where the absence of a device is itself the check.
"""

from __future__ import annotations

import ctypes
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "tllm.h"

from triton_llm import _lib  # noqa: E402


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(tllm_\w+)\s*\(",
                                 text, flags=re.M)))


def test_library_exists_and_loads():
    assert _lib.LIB_PATH.exists(), "build libtllm.so first"
    lib = _lib.load()
    assert lib.tllm_version() >= 100


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared in tllm.h but not exported: {missing}"
    unbound = [n for n in names
               if n not in _lib.SIGNATURES and n != "tllm_last_error_string"]
    assert not unbound, f"exported but without a ctypes signature: {unbound}"


def test_no_undeclared_exports():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)],
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (tllm_\w+)", out))
    assert exported == set(_declared())


def test_status_mapping():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARG, "x")
    with pytest.raises(RuntimeError, match="GPU runtime error"):
        _lib.check(_lib.ERR_CUDA, "x")
    with pytest.raises(RuntimeError, match="No supported GPU runtime found"):
        _lib.check(_lib.ERR_NO_DEVICE, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    _lib.check(_lib.OK)


def test_argument_errors_before_any_device_work():
    lib = _lib.load()
    pb, cb = ctypes.c_size_t(), ctypes.c_size_t()
    # n_head not divisible by n_kv_head -> invalid argument, message set
    st = lib.tllm_gqa_decode_workspace(4, 9, 2, 64, 128, _lib.BF16,
                                       ctypes.byref(pb), ctypes.byref(cb))
    assert st == _lib.ERR_INVALID_ARG
    assert "divisible" in _lib.last_error()
    st = lib.tllm_gqa_decode_workspace(4, 9, 3, 64, 128, _lib.BF16,
                                       ctypes.byref(pb), ctypes.byref(cb))
    assert st == _lib.OK and pb.value > 0 and cb.value == 4 * 9 * 4


def test_mlp_workspace_rejects_unsupported_shapes():
    """tllm_mlp_workspace checks the block's shape rules on the host."""
    lib = _lib.load()
    n = ctypes.c_size_t()
    for args, msg in [((0, 1024, 1024, 2816), "M must be in"),
                      ((65, 1024, 1024, 2816), "M must be in"),
                      ((8, 1024, 1000, 2816), "hidden must be a multiple of 128"),
                      ((8, 1000, 1024, 2816), "attn_dim must be a multiple of 64"),
                      ((8, 1024, 1024, 2800), "ffn must be a multiple of 64")]:
        assert lib.tllm_mlp_workspace(*args, ctypes.byref(n)) == _lib.ERR_INVALID_ARG
        assert msg in _lib.last_error()
    assert lib.tllm_mlp_workspace(8, 1024, 1024, 2816, ctypes.byref(n)) == _lib.OK
    assert n.value > 0 and n.value % 256 == 0


def _has_device():
    n = ctypes.c_int(0)
    return _lib.load().tllm_device_count(ctypes.byref(n)) == 0 and n.value > 0


@pytest.mark.skipif(_has_device(), reason="checks the no-device path")
def test_no_device_raises_reference_message():
    from triton_llm import gpu
    with pytest.raises(RuntimeError, match="No supported GPU runtime found"):
        gpu.allocate((4,))


def test_fault_injection_on_malloc():
    # The injected failure is decided before any CUDA call, so this runs on
    # CPU: the first tllm_malloc of the process must fail with INJECTED.
    code = (
        "import ctypes, sys; sys.path.insert(0, %r);"
        "from triton_llm import _lib; lib = _lib.load();"
        "p = ctypes.c_void_p();"
        "st = lib.tllm_malloc(ctypes.byref(p), 64);"
        "print(st, _lib.last_error())" % str(REPO / "triton-llm_b200"))
    env = dict(os.environ, TLLM_FAULT_INJECT="malloc:1")
    r = subprocess.run([sys.executable, "-c", code], env=env,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    st, msg = r.stdout.strip().split(" ", 1)
    assert int(st) == _lib.ERR_INJECTED
    assert "injected" in msg
