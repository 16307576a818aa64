"""Invariants of the streaming GEMV kernel's launch plan (host arithmetic,
no GPU): every shared-memory region fits the 227 KB opt-in and none overlaps
another, bulk-copy destinations are 16-byte aligned, the split-K cluster gives
every rank work, the grid fits the SMs, and every shape of the benchmarks and
of the tensor-parallel decoders gets a plan (no silent fallback)."""

from __future__ import annotations

import ctypes

import pytest

from dequant_project_b200 import _native

# Kernel constants (csrc/gemv.h).
MAX_SMEM, TILE, NRB, NCW, BAR, X_MAX = 232448, 16, 4, 8, 512, 100 * 1024
NUM_SMS = 148
FIELDS = ("wpl mp ks n_slabs stages n_meta w_pitch xp stage_bytes C KC off_x off_sstep off_sx "
          "off_meta meta_half meta_stride off_red off_bar off_xred off_zero smem grid").split()


def plan(m, n, k, bits, gs):
    out = (ctypes.c_int32 * 23)()
    rc = _native.lib().dqg_stream_plan(m, n, k, bits, gs, NUM_SMS, out, 23)
    return rc, dict(zip(FIELDS, out))


def check(m, n, k, bits, gs):
    rc, p = plan(m, n, k, bits, gs)
    assert rc == 0, (m, n, k, bits, gs, _native.lib().dqg_last_error())
    grouped = gs < k
    pp = 32 // bits
    sc = 4 * p["wpl"] * pp
    gslots = 8 // p["mp"] if grouped else 1
    unit = gslots * gs if grouped else sc
    C, KC = p["C"], p["KC"]
    assert C in (1, 2, 4, 8) and KC % unit == 0 and (C - 1) * KC < k <= C * KC
    assert (m * p["xp"] + 127) // 128 * 128 <= X_MAX
    assert p["xp"] >= 2 * KC and p["xp"] % 128 == 32
    assert 2 <= p["stages"] <= 8 and 2 <= p["n_meta"] <= 8
    assert p["ks"] % unit == 0 or p["ks"] == KC
    assert p["n_slabs"] * p["ks"] >= KC > (p["n_slabs"] - 1) * p["ks"]
    assert p["w_pitch"] >= p["ks"] * bits // 8 and p["w_pitch"] % 16 == 0
    assert p["stage_bytes"] >= TILE * p["w_pitch"] and p["stage_bytes"] % 128 == 0
    groups = KC // gs if grouped else 1
    regions = [
        ("ring", 0, p["stages"] * p["stage_bytes"]),
        ("x", p["off_x"], m * p["xp"]),
        ("sstep", p["off_sstep"], m * (KC // sc) * 4),
        ("sx", p["off_sx"], m * groups * 4),
        ("zero", p["off_zero"], 2 * sc),
        ("xred", p["off_xred"], NRB * C * TILE * m * 4 if C > 1 else 0),
        ("red", p["off_red"], NRB * NCW * TILE * m * 4),
        ("bar", p["off_bar"], BAR),
        ("meta", p["off_meta"], p["n_meta"] * p["meta_stride"]),
    ]
    assert p["smem"] <= MAX_SMEM
    spans = sorted((o, o + size, name) for name, o, size in regions if size)
    for (a0, a1, na), (b0, b1, nb) in zip(spans, spans[1:]):
        assert a1 <= b0, f"{na} [{a0},{a1}) overlaps {nb} [{b0},{b1})"
    assert spans[-1][1] <= p["smem"]
    for name in ("off_x", "off_meta", "off_red", "off_xred", "off_sstep", "off_sx"):
        assert p[name] % 16 == 0, name
    # A tile's metadata buffer holds 16 rows x all K/gs groups (plus the slack
    # of copying from the enclosing 16-byte boundary).
    assert p["off_bar"] % 8 == 0 and p["meta_half"] >= TILE * (k // gs) * 2 + 16
    assert p["meta_stride"] == 2 * p["meta_half"] and p["meta_half"] % 16 == 0
    tiles = -(-n // TILE)
    assert p["grid"] % C == 0 and C <= p["grid"] <= NUM_SMS and p["grid"] // C <= tiles
    return p


FORMATS = [(8, None), (4, 128), (4, 64), (2, 64), (2, 128)]
SWEEP = [(4096, 11008), (11008, 4096), (4096, 4096), (12288, 4096), (4096, 14336),
         (28672, 8192), (8192, 28672), (128256, 4096)]


@pytest.mark.parametrize("m", (1, 2, 3, 4, 5, 8))
@pytest.mark.parametrize("bits,gs", FORMATS)
@pytest.mark.parametrize("n,k", SWEEP)
def test_benchmark_shapes_have_valid_plans(n, k, bits, gs, m):
    check(m, n, k, bits, gs or k)


def _decoder_shapes(hidden, heads, kv, inter, vocab, world):
    d = hidden // heads
    hq, hk = heads // world, kv // world
    units = inter // 128
    ir = -(-units // world) * 128
    return [((hq + 2 * hk) * d, hidden), (hidden, hq * d), (2 * ir, hidden), (hidden, ir),
            (-(-vocab // world), hidden)]


@pytest.mark.parametrize("world", (1, 2, 4, 8))
@pytest.mark.parametrize("model", ("7b", "70b"))
def test_decoder_shapes_have_valid_plans(model, world):
    cfg = (4096, 32, 32, 11008, 32000) if model == "7b" else (8192, 64, 8, 28672, 128256)
    for n, k in _decoder_shapes(*cfg, world):
        for bits, gs in ((4, 128), (2, 64)):
            for m in (1, 8):
                check(m, n, k, bits, gs)


def test_split_k_engages_when_activations_do_not_fit():
    p = check(8, 4096, 11008, 4, 128)           # 8 x 11008 fp16 = 176 KB of activations
    assert p["C"] >= 2
    assert check(1, 4096, 11008, 4, 128)["C"] == 1
    assert check(8, 8192, 28672, 4, 128)["C"] >= 4


def test_rejects_bad_arguments():
    out = (ctypes.c_int32 * 23)()
    lib = _native.lib()
    assert lib.dqg_stream_plan(9, 64, 256, 4, 128, NUM_SMS, out, 23) != 0
    assert lib.dqg_stream_plan(1, 64, 250, 4, 128, NUM_SMS, out, 23) != 0
    assert lib.dqg_stream_plan(1, 64, 256, 3, 128, NUM_SMS, out, 23) != 0
    assert lib.dqg_stream_plan(1, 64, 256, 4, 128, NUM_SMS, out, 10) != 0
