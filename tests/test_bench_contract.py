"""The reference arm of bench.py (CPU only) prints one JSON line with the
contract's keys, on the GPU arm's metric (decode tokens/s), unit and config."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    b = json.loads(lines[0])
    sys.path.insert(0, str(ROOT))
    import bench
    assert b["impl"] == "reference" and b["metric"] == bench.METRIC and b["unit"] == bench.UNIT
    assert b["config"] == bench.workload_config(1)
    assert b["steps"] >= 1 and b["warmup"] == 3 and b["higher_is_better"] is True
    assert b["scaling"] == "strong"
    assert b["value"] > 0 and b["cpu_baseline"]["value"] == b["value"]
    assert b["cpu_baseline"]["kind"] == "port" and b["cpu_baseline"]["cores"] >= 1
    assert b["e2e"] == {"value": b["value"], "unit": b["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_launch_count_follows_the_step():
    sys.path.insert(0, str(ROOT))
    import bench
    from dequant_project_b200.decoder import LLAMA2_7B
    # Per layer: two norms (the all-reduces run inside them at world > 1),
    # QKV, O, gate/up + SwiGLU and down GEMVs, RoPE + KV append, attention.
    assert bench.decode_launches(LLAMA2_7B, 1) == 32 * 8 + 2
    assert bench.decode_launches(LLAMA2_7B, 8) == 32 * 8 + 2
