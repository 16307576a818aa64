"""The C-ABI library: loads, exports every declared symbol, and rejects bad
arguments before touching the GPU (runs on CPU-only hosts)."""

from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import ROOT
from dequant_project_b200 import _native, dequant_cuda

HEADER = ROOT / "include" / "dequant_b200.h"


def declared_symbols():
    return sorted(set(re.findall(r"\b(dqg_[a-z_]+)\s*\(", HEADER.read_text())))


def test_header_declares_exactly_the_exported_set():
    assert declared_symbols() == sorted(_native.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.dqg_version() == 100


def _gemv_rc(**kw):
    a = dict(x=16, qw=16, s=2, z=None, y=2, M=1, N=64, K=512, bits=4, g=128, sym=1, inter=0)
    a.update(kw)
    lib = _native.lib()
    return lib.dqg_gemv(a["x"], a["qw"], a["s"], a["z"], a["y"], a["M"], a["N"], a["K"],
                        a["bits"], a["g"], a["sym"], a["inter"], None)


@pytest.mark.parametrize("kw,msg", [
    (dict(M=0), "1 <= M <= 8"),
    (dict(M=9), "1 <= M <= 8"),
    (dict(bits=3), "bits must be 2, 4 or 8"),
    (dict(g=0), "group_size must be positive"),
    (dict(K=500), "not divisible by group_size"),
    (dict(sym=0), "symmetric=false requires zeros"),
    (dict(z=2), "symmetric=true takes no zeros"),
    (dict(bits=2, g=32, K=512), "this excludes INT2 with group_size 32"),
    (dict(x=8), "x must be 16-byte aligned"),
    (dict(qw=8), "qweight must be 16-byte aligned"),
    (dict(N=0), "at least one row"),
])
def test_gemv_rejects_bad_arguments_without_a_gpu(kw, msg):
    assert _gemv_rc(**kw) == 1
    assert msg in _native.lib().dqg_last_error().decode()


def test_dequantize_rejects_bad_group():
    lib = _native.lib()
    # INT4 with group 4: not a whole number of 8-code words.
    rc = lib.dqg_dequantize(16, 2, None, 16, 64, 512, 4, 4, 1, 0, None)
    assert rc == 1 and b"values per uint32 word" in lib.dqg_last_error()


def test_binding_validates_like_the_reference():
    """RuntimeError with the reference's message, before any CUDA work."""
    x = torch.zeros(1, 512, dtype=torch.float16)
    qw = torch.zeros(64, 64, dtype=torch.int32)
    s = torch.zeros(64, 4, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        dequant_cuda.gemv(x, qw, s, None, 4, 128, True, False)
    with pytest.raises(RuntimeError, match="qweight must be a CUDA tensor"):
        dequant_cuda.dequantize(qw, s, None, 4, 128, True, False, 512)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        dequant_cuda.add_one(torch.ones(4))
    with pytest.raises(RuntimeError, match="bits must be 2, 4 or 8"):
        dequant_cuda.dequantize(qw, s, None, 3, 128, True, False, 512)


def test_starved_diagnostic_rejects_bad_limits_without_a_gpu():
    lib = _native.lib()
    for wait_ns in (0, 10, 2_000_000_000):
        rc = lib.dqg_debug_gemv_starved(16, 16, 16, 16, 16, 1, 64, 512, 4, 128, 0, 0, wait_ns,
                                        None)
        assert rc == 1 and b"wait_ns must be in" in lib.dqg_last_error()


def test_weight_prefetch_switch_round_trips():
    lib = _native.lib()
    prev = lib.dqg_set_weight_prefetch(0)
    try:
        assert lib.dqg_set_weight_prefetch(1) == 0
        assert lib.dqg_set_weight_prefetch(1) == 1
    finally:
        lib.dqg_set_weight_prefetch(prev)


def test_l2_spans_layout_and_limits():
    """dqg_l2_spans as ctypes lays out like the C struct (8 pointers, 8 sizes,
    a count); at most 8 ranges, empty ranges dropped."""
    s = _native.L2Spans.of([(0x1000, 4096), (0x9000, 0), (0x20000, 64)])
    assert ctypes.sizeof(_native.L2Spans) == 8 * 8 + 8 * 8 + 8
    assert s.n == 2 and s.ptr[1] == 0x20000 and s.bytes[0] == 4096
    with pytest.raises(ValueError):
        _native.L2Spans.of([(0x1000, 16)] * 9)
    assert "dqg_l2_spans" in HEADER.read_text()
