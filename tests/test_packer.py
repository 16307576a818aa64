"""The product's packer (torch): bit-exact with the reference, and the
reference's packer properties (scripts/test_packer.py:47-155) as pytest."""

from __future__ import annotations

import pytest
import torch

from conftest import bench_inputs, load_golden, sha16, small_inputs
from dequant_project_b200.packer import (QuantConfig, dequantize, pack, quantize,
                                         quantize_tensor, unpack)

BITS = (2, 4, 8)
LAYOUTS = ("sequential", "interleaved")
GROUPS = (32, 64, 128, 256, None)
CASES = load_golden("packer_cases.json")["cases"]


@pytest.fixture(scope="module")
def inputs():
    gauss, skew, x = small_inputs(0)
    return {"gauss": gauss, "skew": skew, "x": x}


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['bits']}b-{c['layout'][:3]}-"
                         f"{'sym' if c['symmetric'] else 'asym'}-g{c['group_size']}-{c['input']}")
def test_bit_exact_with_reference(case, inputs):
    cfg = QuantConfig(case["bits"], case["group_size"], case["symmetric"], case["layout"])
    pw = quantize_tensor(inputs[case["input"]], cfg)
    assert sha16(pw.qweight) == case["qweight"]
    assert sha16(pw.scales) == case["scales"]
    assert (pw.zeros is None) if case["zeros"] is None else sha16(pw.zeros) == case["zeros"]
    assert sha16(dequantize(pw)) == case["deq"]


def test_bit_exact_at_benchmark_shape():
    case = next(c for c in load_golden("known_answers.json")["cases"]
                if c["N"] == 4096 and c["K"] == 4096)
    w, _ = bench_inputs(4096, 4096)
    pw = quantize_tensor(w, QuantConfig(4, 128, False))
    assert (sha16(pw.qweight), sha16(pw.scales), sha16(pw.zeros)) == \
        (case["qweight"], case["scales"], case["zeros"])


@pytest.mark.parametrize("bits", BITS)
@pytest.mark.parametrize("layout", LAYOUTS)
def test_pack_roundtrip(bits, layout):
    torch.manual_seed(0)
    cfg = QuantConfig(bits=bits, layout=layout)
    q = torch.randint(0, cfg.qmax + 1, (8, 512), dtype=torch.int32)
    assert torch.equal(unpack(pack(q, cfg), cfg, 512), q)


@pytest.mark.parametrize("bits", BITS)
@pytest.mark.parametrize("sym", (True, False))
@pytest.mark.parametrize("gs", GROUPS)
def test_error_within_bound(bits, sym, gs):
    torch.manual_seed(0)
    w = torch.randn(64, 512, dtype=torch.float16)
    cfg = QuantConfig(bits=bits, group_size=gs, symmetric=sym)
    pw = quantize_tensor(w, cfg)
    err = (dequantize(pw).float() - w.float()).abs()
    step = pw.scales.float().repeat_interleave(cfg.effective_group_size(512), dim=1)
    bound = step * (0.5 if sym else 1.0) + 1e-3
    assert (err / bound).max().item() <= 1.0


def test_error_monotonic_in_bits_and_group():
    torch.manual_seed(0)
    w = torch.randn(64, 512, dtype=torch.float16)
    e_bits = [(dequantize(quantize_tensor(w, QuantConfig(b, 128))).float() - w.float())
              .abs().mean().item() for b in BITS]
    assert all(a > b for a, b in zip(e_bits, e_bits[1:]))
    e_grp = [(dequantize(quantize_tensor(w, QuantConfig(4, g))).float() - w.float())
             .abs().mean().item() for g in GROUPS]
    assert all(a < b for a, b in zip(e_grp, e_grp[1:]))


def test_asymmetric_wins_on_skew():
    torch.manual_seed(0)
    w = (torch.rand(64, 512) * 0.5 + 2.0).to(torch.float16)
    e_sym = (dequantize(quantize_tensor(w, QuantConfig(4, 128, True))).float() - w.float()).abs().mean()
    e_asym = (dequantize(quantize_tensor(w, QuantConfig(4, 128, False))).float() - w.float()).abs().mean()
    assert e_asym < e_sym


@pytest.mark.parametrize("bits", BITS)
def test_layout_does_not_change_values(bits):
    torch.manual_seed(0)
    w = torch.randn(64, 512, dtype=torch.float16)
    a = dequantize(quantize_tensor(w, QuantConfig(bits, 128, True, "sequential")))
    b = dequantize(quantize_tensor(w, QuantConfig(bits, 128, True, "interleaved")))
    assert torch.equal(a, b)


@pytest.mark.parametrize("n,k", [(3072, 3072), (1024, 3072), (8192, 3072), (3072, 8192)])
def test_error_matches_prediction_on_real_shapes(n, k):
    torch.manual_seed(0)
    w = torch.randn(n, k, dtype=torch.float16) * 0.02
    pw = quantize_tensor(w, QuantConfig(4, 128, True))
    err = (dequantize(pw).float() - w.float()).abs().mean().item()
    ratio = err / (pw.scales.float().mean().item() / 4)
    assert 0.85 <= ratio <= 1.15


def test_config_validation():
    with pytest.raises(ValueError):
        QuantConfig(bits=3)
    with pytest.raises(ValueError):
        QuantConfig(layout="zigzag")
    with pytest.raises(ValueError):
        QuantConfig(group_size=0)
    with pytest.raises(ValueError):
        quantize(torch.zeros(4, 100, dtype=torch.float16), QuantConfig(4, 64))
    cfg = QuantConfig(4, None, False)
    assert cfg.per_pack == 8 and cfg.qmax == 15 and cfg.bias == 8
    assert cfg.groups_for(4096) == 1 and cfg.effective_group_size(4096) == 4096
