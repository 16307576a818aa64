"""Byte model: the algorithmic bytes that every roofline number divides by."""

from __future__ import annotations

import pytest

from dequant_project_b200.byte_model import gemv_bytes, gemv_flops, measured_peaks


@pytest.mark.parametrize("n,k,bits,g,sym,m,mb", [
    # Values of the bytes-moved table for the benchmark configurations.
    (4096, 11008, 8, None, True, 1, 45.13),
    (4096, 11008, 8, None, True, 8, 45.34),
    (4096, 11008, 4, 128, False, 1, 23.98),
    (4096, 11008, 4, 128, False, 8, 24.20),
    (4096, 11008, 2, 64, False, 1, 14.12),
    (4096, 11008, 2, 64, False, 4, 14.21),
    (4096, 4096, 4, 128, False, 1, 8.93),
    (28672, 8192, 4, 128, False, 1, 124.85),
    (128256, 4096, 4, 128, False, 1, 279.35),
])
def test_gemv_bytes(n, k, bits, g, sym, m, mb):
    assert gemv_bytes(n, k, bits, g, sym, m) / 1e6 == pytest.approx(mb, abs=0.01)


def test_transposed_grouped_shapes_move_the_same_bytes():
    # Groups run along K and are flat-contiguous, so N x K and K x N hold the
    # same number of groups; the x read and y write swap roles.
    for m in (1, 4, 8):
        assert gemv_bytes(4096, 11008, 4, 128, False, m) == gemv_bytes(11008, 4096, 4, 128, False, m)


def test_flops_and_peaks():
    assert gemv_flops(4096, 4096, 1) == 2 * 4096 * 4096
    p = measured_peaks()
    assert p["hbm_gbs"] > 1000 and p["source"] in ("measured", "fallback")
