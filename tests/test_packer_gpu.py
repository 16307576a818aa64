"""The packer on CUDA tensors (the GPU packer used to build models on the
device) is bit-exact with the numpy oracle, which is pinned to the reference's
golden vectors: same codes, words, scales and zero-points for every format,
including constant groups and skewed weights."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dequant_project_b200.packer import QuantConfig, quantize_tensor
from oracle import packer_np as P

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.mark.parametrize("gs", (32, 64, 128, None))
@pytest.mark.parametrize("sym", (True, False), ids=("sym", "asym"))
@pytest.mark.parametrize("layout", ("sequential", "interleaved"))
@pytest.mark.parametrize("bits", (2, 4, 8))
def test_cuda_packer_bit_exact_with_oracle(bits, layout, sym, gs):
    torch.manual_seed(bits * 7 + (gs or 0))
    gauss = torch.randn(257, 1024, dtype=torch.float16) * 0.02
    skew = (torch.rand(257, 1024) * 0.5 + 2.0).to(torch.float16)
    gauss[5, :256] = 0.125                           # constant groups
    for w in (gauss, skew):
        pw = quantize_tensor(w.cuda(), QuantConfig(bits, gs, sym, layout))
        qw, s, z = P.quantize_tensor(w.numpy(), bits, gs, sym, layout)
        assert np.array_equal(pw.qweight.cpu().numpy().view(np.uint32), qw.view(np.uint32))
        assert np.array_equal(pw.scales.cpu().numpy().view(np.uint16), s.view(np.uint16))
        if sym:
            assert pw.zeros is None and z is None
        else:
            assert np.array_equal(pw.zeros.cpu().numpy().view(np.uint16), z.view(np.uint16))
