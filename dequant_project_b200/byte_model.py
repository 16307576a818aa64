"""Algorithmic byte counts and roofline denominators for the packed GEMV path.

Extends KrishnaI2424/Dequant_Project ``dequant/byte_model.py`` (``_quant_bytes``
:165-176, and the per-call bytes of scripts/bench_dequant_kernel.py:156) into
the per-call roofline that every benchmark row reports against:

    B(N, K, M) = N*K*bits/8                   packed codes
               + N*(K/g)*2*(1 + asym)        fp16 scales (+ zero-points)
               + M*K*2                        fp16 activations read
               + M*N*2                        fp16 outputs written

with g = K for per-channel formats. (The reference's ``_quant_bytes`` counts no
metadata at all for per-channel, undercounting by 2N bytes; this counts it.)
"""

from __future__ import annotations

import json
from pathlib import Path

# Fallback denominators when the pool's measured peaks are absent (an earlier
# measurement of a B200 on this pool): HBM copy GB/s and dense bf16 TFLOP/s.
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
NOMINAL_HBM_GBS = 8000.0


def gemv_bytes(n: int, k: int, bits: int, group_size, symmetric: bool, m: int) -> int:
    """Bytes one fused dequant+GEMV call must move at minimum."""
    g = k if group_size is None else group_size
    meta = n * (k // g) * 2 * (1 if symmetric else 2)
    return n * k * bits // 8 + meta + m * k * 2 + m * n * 2


def gemv_flops(n: int, k: int, m: int) -> int:
    return 2 * m * n * k


def dequantize_bytes(n: int, k: int, bits: int, group_size, symmetric: bool) -> int:
    """Bytes of the materialising dequantize: packed read + fp16 [N, K] write."""
    g = k if group_size is None else group_size
    return n * k * bits // 8 + n * (k // g) * 2 * (1 if symmetric else 2) + n * k * 2


def measured_peaks(path: Path | None = None) -> dict:
    """Peaks measured on this pool's B200s (MEASURED_PEAKS.json at the repo root).

    Returns {"hbm_gbs", "bf16_tflops", "source"} with source "measured" or
    "fallback".
    """
    p = path or Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
                "bf16_tflops_sustained": 1400.0, "source": "fallback"}
