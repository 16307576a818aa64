"""Build the reference's own CUDA extension, unmodified, for B200 (sm_100a).

    python baseline/build_reference_kernel.py [REFERENCE_ROOT]

Compiles KrishnaI2424/Dequant_Project's ``kernels/smoke.cu``,
``kernels/dequant_gemv.cu`` and ``kernels/bindings.cpp`` (the sources its
``setup.py:28-42`` builds) where they lie in the reference checkout
(REFERENCE_ROOT, or the DEQUANT_REFERENCE_ROOT environment variable), with
torch's extension builder and ``-gencode arch=compute_100a,code=sm_100a`` in
place of the reference's sm_75 / sm_120 targets. The module lands in
``baseline/_ref/ext/`` (not tracked; it travels with the repository to the GPU
box), where ``bench.py`` loads it to time the reference kernel beside this
library's on the same shapes. Nothing of the reference is copied into the
repository.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "ext"
NAME = "dequant_cuda_ref"


def build(reference_root: str) -> Path:
    # torch's builder adds -gencode flags for this arch list; B200 only.
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    kernels = Path(reference_root) / "kernels"
    sources = [str(kernels / f) for f in ("smoke.cu", "dequant_gemv.cu", "bindings.cpp")]
    for s in sources:
        if not Path(s).exists():
            raise SystemExit(f"missing reference source {s}")
    OUT.mkdir(parents=True, exist_ok=True)
    load(name=NAME, sources=sources, build_directory=str(OUT), verbose=False,
         extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a", "-O3"],
         extra_cflags=["-O3"])
    so = next(OUT.glob(f"{NAME}*.so"))
    return so


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DEQUANT_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: build_reference_kernel.py REFERENCE_ROOT")
    print(build(root))
