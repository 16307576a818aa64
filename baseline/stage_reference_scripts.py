"""Stage the reference's own kernel test scripts to run through this library.

    python baseline/stage_reference_scripts.py [REFERENCE_ROOT]

Copies KrishnaI2424/Dequant_Project's ``dequant/`` package and its
``scripts/test_dequant_kernel.py`` and ``scripts/test_quant_linear.py``,
unmodified, from the reference checkout (REFERENCE_ROOT, or the
DEQUANT_REFERENCE_ROOT environment variable) into ``baseline/_ref/src/``
(not tracked; it travels with the repository to the GPU box), and writes the
one-line ``dequant_cuda.py`` shim of INTEGRATION.md at that root in place of
the reference's compiled extension. ``tests/test_reference_scripts_gpu.py``
then runs both scripts as the reference's maintainers do.
"""

from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "_ref" / "src"
SCRIPTS = ("test_dequant_kernel.py", "test_quant_linear.py")
SHIM = "from dequant_project_b200.dequant_cuda import add_one, gemv, dequantize  # noqa: F401\n"


def stage(reference_root: str) -> Path:
    root = Path(reference_root)
    if DEST.exists():
        shutil.rmtree(DEST)
    (DEST / "scripts").mkdir(parents=True)
    shutil.copytree(root / "dequant", DEST / "dequant",
                    ignore=shutil.ignore_patterns("__pycache__"))
    for name in SCRIPTS:
        shutil.copy2(root / "scripts" / name, DEST / "scripts" / name)
    (DEST / "dequant_cuda.py").write_text(SHIM)
    return DEST


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DEQUANT_REFERENCE_ROOT")
    if not ref:
        raise SystemExit("usage: stage_reference_scripts.py REFERENCE_ROOT")
    print(stage(ref))
