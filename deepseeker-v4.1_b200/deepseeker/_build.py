"""Build libdeepseeker_b200.so (all CUDA sources, sm_100a) in-tree.

    python -m deepseeker._build          (from deepseeker-v4.1_b200/)

Objects go to ``deepseeker-v4.1_b200/_build/`` and the shared library to
``deepseeker-v4.1_b200/deepseeker/_lib/libdeepseeker_b200.so``.  A source is
recompiled only when it or a header is newer than its object.  The dequant
kernels must stay bit-exact, so no fast-math / flush-to-zero flags are used.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]          # deepseeker-v4.1_b200/
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = PKG_ROOT / "_build"
LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = LIB_DIR / "libdeepseeker_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
          "-I", str(INCLUDE), "-I", str(CSRC)]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, hdr_mtime: float) -> bool:
    if not obj.exists():
        return True
    m = obj.stat().st_mtime
    return m < src.stat().st_mtime or m < hdr_mtime


def _compile(src: Path, obj: Path) -> None:
    cmd = [NVCC, *ARCH, *CFLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")


def build(verbose: bool = True, jobs: int | None = None) -> Path:
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if _stale(o, s, hdr_mtime)]
    if todo:
        if verbose:
            print(f"[deepseeker_b200] compiling {len(todo)} source(s) for sm_100a", flush=True)
        with ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda so: _compile(*so), todo))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"[deepseeker_b200] linked {LIB_PATH}", flush=True)
    return LIB_PATH


if __name__ == "__main__":
    build()
    sys.exit(0)
