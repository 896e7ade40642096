"""Build libtllm.so (sm_100a) from the CUDA sources in this directory.

    python triton-llm_b200/csrc/build.py [--force] [-j N]

Each ``*.cu`` file is compiled by nvcc for ``-gencode
arch=compute_100a,code=sm_100a`` into ``triton-llm_b200/_build/`` and the
objects are linked into ``triton-llm_b200/triton_llm/libtllm.so`` with the
CUDA runtime linked statically, so the library only needs the NVIDIA driver
at run time. Objects are rebuilt when their source or any header changed.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
REPO = PKG_ROOT.parent
BUILD = PKG_ROOT / "_build"
OUT = PKG_ROOT / "triton_llm" / "libtllm.so"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-O3",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"),
                 "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put it on PATH)")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC),
           "-DTLLM_BUILD=1", "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)


def build(force: bool = False, jobs: int | None = None,
          verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objs)
            if force or _stale(o, s, headers)]
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = [ex.submit(_compile, s, o, verbose) for s, o in todo]
            for f in futs:
                f.result()
    if force or todo or not OUT.exists() or any(
            o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs), "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, OUT)
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true",
                    help="print ptxas register/spill/smem usage")
    a = ap.parse_args()
    out = build(force=a.force, jobs=a.j, verbose=a.verbose)
    print(out)


if __name__ == "__main__":
    main()
