"""Materialising dequantize on the GPU: bit-exact with the oracle (and so with
the reference packer) over every bits x layout x symmetry x group format
(scripts/test_dequant_kernel.py:63-89), plus add_one (:56-60)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dequant_project_b200 import dequant_cuda
from oracle import packer_np as P

pytestmark = pytest.mark.gpu

BITS = (2, 4, 8)
LAYOUTS = ("sequential", "interleaved")
GROUPS = (32, 64, 128, 256, None)


@pytest.fixture(scope="module")
def weights():
    torch.manual_seed(0)
    n, k = 1024, 3072
    gauss = (torch.randn(n, k, dtype=torch.float16) * 0.02).numpy()
    skew = (torch.rand(n, k) * 0.5 + 2.0).to(torch.float16).numpy()
    return {"gauss": gauss, "skew": skew}


@pytest.mark.parametrize("gs", GROUPS)
@pytest.mark.parametrize("sym", (True, False), ids=("sym", "asym"))
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("bits", BITS)
def test_dequantize_bit_exact(weights, bits, layout, sym, gs):
    tags = ("gauss",) if sym else ("gauss", "skew")
    for tag in tags:
        w = weights[tag]
        k = w.shape[1]
        qw, s, z = P.quantize_tensor(w, bits, gs, sym, layout)
        want = P.dequantize(qw, s, z, bits, gs, sym, layout, k)
        dev = [None if a is None else torch.from_numpy(a).cuda() for a in (qw, s, z)]
        got = dequant_cuda.dequantize(*dev, bits, gs or k, sym, layout == "interleaved", k)
        got = got.cpu().numpy()
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), \
            f"{tag}: {(got.view(np.uint16) != want.view(np.uint16)).sum()} words differ"


@pytest.mark.parametrize("n,k,bits,gs", [(1, 16, 2, 16), (3, 40, 8, 8), (5, 24, 4, 8),
                                         (129, 96, 2, 32), (2, 4096, 8, None)])
def test_dequantize_odd_shapes(n, k, bits, gs):
    rng = np.random.default_rng(n * k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    for sym in (True, False):
        qw, s, z = P.quantize_tensor(w, bits, gs, sym, "sequential")
        want = P.dequantize(qw, s, z, bits, gs, sym, "sequential", k)
        dev = [None if a is None else torch.from_numpy(a).cuda() for a in (qw, s, z)]
        got = dequant_cuda.dequantize(*dev, bits, gs or k, sym, False, k).cpu().numpy()
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def test_add_one():
    out = dequant_cuda.add_one(torch.ones(4, device="cuda"))
    assert torch.equal(out, torch.full((4,), 2.0, device="cuda"))
    big = torch.arange(1 << 20, dtype=torch.float32, device="cuda")
    assert torch.equal(dequant_cuda.add_one(big), big + 1)
