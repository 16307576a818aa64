"""Build libdequant_b200.so in-tree (sm_100a only).

    python -m dequant_project_b200.build [--force] [--verbose-ptxas]

Each ``csrc/*.cu`` is compiled by nvcc for ``arch=compute_100a,code=sm_100a``
with ``-lineinfo`` and linked into ``dequant_project_b200/libdequant_b200.so``
next to this file (static CUDA runtime, no torch dependency). The shared
library is the product's C ABI (include/dequant_b200.h); the Python package
loads it with ctypes.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT = PKG / "libdequant_b200.so"
OBJ_DIR = PKG / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(paths) -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(paths) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    srcs = sources()
    if not force and not _stale(srcs):
        return OUT
    OBJ_DIR.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--verbose-ptxas" in sys.argv))
