"""Build recipe for the C oracle (TEST INFRASTRUCTURE ONLY).

    python oracle/build.py        ->  oracle/_build/liboracle_gemv.so

gcc with OpenMP; x86-64-v3 (AVX2/FMA/F16C) so that the library built here runs
on the GPU box's host cores as well. No reference sources are compiled: the
reference's CPU path is Python/torch, so this is our restatement of it.
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_build"
LIB = OUT_DIR / "liboracle_gemv.so"
SRC = HERE / "cpu_gemv.c"


def build(force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared",
           "-o", str(LIB), str(SRC)]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
