"""Pin the CPU oracle to the reference: every golden vector must match.

The golden files were produced by the reference's own packer and CPU GEMV path
(tests/golden/make_golden.py). The numpy restatement must reproduce qweight,
scales, zeros and the dequantized weight bit for bit; its GEMV (and the C
restatement's) must agree with the reference's F.linear output to fp32
summation-order noise.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import bench_inputs, fp16_from_hex, load_golden, sha16, small_inputs
from oracle import native
from oracle import packer_np as P

CASES = load_golden("packer_cases.json")["cases"]
BIG = load_golden("known_answers.json")["cases"]


def _case_id(c):
    return (f"{c['bits']}b-{c['layout'][:3]}-{'sym' if c['symmetric'] else 'asym'}"
            f"-g{c['group_size']}-{c['input']}")


@pytest.fixture(scope="module")
def inputs():
    gauss, skew, x = small_inputs(0)
    return {"gauss": gauss.numpy(), "skew": skew.numpy(), "x": x.numpy()}


@pytest.mark.parametrize("case", CASES, ids=_case_id)
def test_numpy_oracle_bit_exact(case, inputs):
    w = inputs[case["input"]]
    qw, s, z = P.quantize_tensor(w, case["bits"], case["group_size"], case["symmetric"],
                                 case["layout"])
    assert sha16(qw) == case["qweight"]
    assert sha16(s) == case["scales"]
    assert (z is None) if case["zeros"] is None else sha16(z) == case["zeros"]
    deq = P.dequantize(qw, s, z, case["bits"], case["group_size"], case["symmetric"],
                       case["layout"], w.shape[1])
    assert sha16(deq) == case["deq"]
    # unpack inverts pack exactly
    codes, _, _ = P.quantize(w, case["bits"], case["group_size"], case["symmetric"])
    assert np.array_equal(P.unpack(qw, case["bits"], case["layout"], w.shape[1]), codes)


@pytest.mark.parametrize("case", [c for c in CASES if "y_fp16_hex" in c], ids=_case_id)
def test_oracle_gemv_matches_reference_path(case, inputs):
    w, x = inputs["gauss"], inputs["x"]
    qw, s, z = P.quantize_tensor(w, case["bits"], case["group_size"], case["symmetric"],
                                 case["layout"])
    yref = fp16_from_hex(case["y_fp16_hex"], (8, 64))
    y = P.gemv_ref(x, qw, s, z, case["bits"], case["group_size"], case["symmetric"],
                   case["layout"])
    assert P.max_rel_err(y, yref) <= 2e-3
    # at most one fp16 ulp apart elementwise: the only difference is summation order
    assert np.abs(y.astype(np.float32) - yref.astype(np.float32)).max() <= \
        np.abs(yref.astype(np.float32)).max() * 2 ** -10
    gs = case["group_size"] or w.shape[1]
    yc = native.gemv(x, qw, s, z, case["bits"], gs, case["symmetric"],
                     case["layout"] == "interleaved")
    assert P.max_rel_err(yc, yref) <= 2e-3
    deq_c = native.dequantize(qw, s, z, case["bits"], gs, case["symmetric"],
                              case["layout"] == "interleaved", w.shape[1])
    assert sha16(deq_c) == case["deq"]


@pytest.mark.parametrize("case", BIG, ids=lambda c: f"{c['N']}x{c['K']}-int{c['bits']}-g{c['group_size']}")
def test_oracle_known_answers_at_benchmark_shapes(case):
    w, x = bench_inputs(case["N"], case["K"])
    assert sha16(w) == case["w"]
    w, x = w.numpy(), x.numpy()
    qw, s, z = P.quantize_tensor(w, case["bits"], case["group_size"], case["symmetric"],
                                 case["layout"])
    assert sha16(qw) == case["qweight"]
    assert sha16(s) == case["scales"]
    assert (z is None) if case["zeros"] is None else sha16(z) == case["zeros"]
    gs = case["group_size"] or case["K"]
    y = native.gemv(x, qw, s, z, case["bits"], gs, case["symmetric"], False)
    yref = fp16_from_hex(case["y_fp16_hex"], (1, case["N"]))
    assert P.max_rel_err(y, yref) <= 2e-3
    assert (y.view(np.uint16) == yref.view(np.uint16)).mean() > 0.99


def test_criterion_flags_a_planted_error(inputs):
    """A wrong value planted in the oracle's output must fail the kernel criterion."""
    w, x = inputs["gauss"], inputs["x"]
    qw, s, z = P.quantize_tensor(w, 4, 128, False, "sequential")
    we = P.exact_weight(qw, s, z, 4, 128, False, "sequential", 512)
    ref = x.astype(np.float32) @ we.T
    y = ref.astype(np.float16)
    err, tol = P.gemv_criterion(y, ref, np.abs(we), np.abs(x.astype(np.float32)))
    assert (err <= tol).all()
    y[3, 7] = np.float16(float(y[3, 7]) + 0.05)
    err, tol = P.gemv_criterion(y, ref, np.abs(we), np.abs(x.astype(np.float32)))
    assert int((err > tol).sum()) == 1 and err[3, 7] > tol[3, 7]
