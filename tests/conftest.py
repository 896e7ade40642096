"""Shared pytest setup.

* registers the ``gpu`` marker (tests that launch CUDA kernels; run on a
  B200 with ``-m gpu``, skipped from ``-m "not gpu"`` CPU runs);
* puts the product package directory (``triton-llm_b200/``) and the repo
  root (for ``oracle``) on ``sys.path``;
* ``golden(name)`` loads a committed fixture from ``tests/golden/``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "triton-llm_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(PKG), str(REPO), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (sm_100a) and the built libtllm.so")


_cache: dict[str, dict] = {}


def load_golden(name: str) -> dict:
    if name not in _cache:
        path = GOLDEN / f"{name}.npz"
        if not path.exists():
            pytest.skip(f"golden fixture {path.name} not generated")
        with np.load(path) as z:
            _cache[name] = {k: z[k] for k in z.files}
    return _cache[name]


@pytest.fixture
def golden():
    return load_golden
