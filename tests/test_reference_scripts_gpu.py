"""The reference's own kernel test scripts, unmodified, through the drop-in
shim: ``scripts/test_dequant_kernel.py`` (bit-exact dequantize over every
format, the GEMV criterion at M = 1, 2, 3, 8, the negative control, graph
capture) and ``scripts/test_quant_linear.py`` (gemv reshape, QuantLinear,
quantize_model, graph capture) import ``dequant_cuda`` from their project root,
where the one-line shim of INTEGRATION.md forwards to this library. Staged by
baseline/stage_reference_scripts.py (skipped when not staged)."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SRC = ROOT / "baseline" / "_ref" / "src"


@pytest.mark.skipif(not (SRC / "scripts").exists(),
                    reason="reference scripts not staged (baseline/stage_reference_scripts.py)")
@pytest.mark.parametrize("script", ("test_dequant_kernel.py", "test_quant_linear.py"))
def test_reference_script_passes_through_the_shim(script):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT), env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, str(SRC / "scripts" / script)], cwd=SRC, env=env,
                       capture_output=True, text=True, timeout=1200)
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0, tail
    assert "ALL PASS" in r.stdout, tail
