"""Fused dequant + GEMV on the GPU against the CPU oracle.

Two criteria, both from the reference:
  * elementwise ``|y - ref| <= 2^-11 |ref| + 2^-20 (|W| @ |x|)`` with ref the
    product of the exact fp32 weight (q - off) * scale
    (scripts/test_dequant_kernel.py:92-122);
  * max relative error <= 2e-3 (max|y - y_ref| / max|y_ref|) against the
    reference CPU path ``F.linear(x, packer.dequantize(pw))``.
Formats, shapes, batch sizes, the ragged INT2 case, the rejections, the
negative control and graph capture follow scripts/test_dequant_kernel.py.
All GPU work goes through the C ABI (dequant_cuda -> libdequant_b200.so).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bench_inputs, fp16_from_hex, load_golden
from dequant_project_b200 import _native, dequant_cuda
from dequant_project_b200.packer import QuantConfig, quantize_tensor
from oracle import native
from oracle import packer_np as P

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def pack_np(w_np, bits, gs, sym, layout):
    return P.quantize_tensor(w_np, bits, gs, sym, layout)


def to_dev(*arrays, dev="cuda"):
    return [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrays]


def gpu_gemv(x, qw, s, z, bits, gs, sym, layout):
    xd, qd, sd, zd = to_dev(x, qw, s, z)
    y = dequant_cuda.gemv(xd, qd, sd, zd, bits, gs, sym, layout == "interleaved")
    return y.cpu().numpy()


def check_against_oracle(x, qw, s, z, bits, gs, sym, layout, y, exact_criterion=True):
    """Assert both criteria; returns (worst err/tol, max rel err)."""
    k = x.shape[1]
    gsz = gs or k
    yref = native.gemv(x, qw, s, z, bits, gsz, sym, layout == "interleaved")
    rel = P.max_rel_err(y, yref)
    assert rel <= REL_TOL, f"max rel err {rel:.3e} vs reference path"
    head = None
    if exact_criterion:
        we = P.exact_weight(qw, s, z, bits, gs, sym, layout, k).astype(np.float64)
        xf = x.astype(np.float64)
        ref = xf @ we.T
        err, tol = P.gemv_criterion(y, ref, np.abs(we), np.abs(xf))
        head = float((err / tol).max())
        assert (err <= tol).all(), f"{int((err > tol).sum())} elements over tolerance, worst {head:.2f}x"
    return head, rel


def run_case(n, k, bits, gs, sym, layout, m, seed=0, w_scale=0.02):
    torch.manual_seed(seed)
    w = (torch.randn(n, k, dtype=torch.float16) * w_scale).numpy()
    x = torch.randn(m, k, dtype=torch.float16).numpy()
    qw, s, z = pack_np(w, bits, gs, sym, layout)
    y = gpu_gemv(x, qw, s, z, bits, gs or k, sym, layout)
    return check_against_oracle(x, qw, s, z, bits, gs, sym, layout, y)


# The reference gate's formats and shapes (scripts/test_dequant_kernel.py:137-146).
GEMV_FORMATS = [
    (4, 128, True, "sequential"), (4, 128, False, "sequential"),
    (4, 128, True, "interleaved"), (4, 128, False, "interleaved"),
    (8, 128, True, "sequential"), (8, 128, True, "interleaved"),
    (4, None, True, "sequential"),
]
GEMV_SHAPES = [(3072, 3072), (1024, 3072), (8192, 3072), (3072, 8192)]


@pytest.mark.parametrize("m", (1, 2, 3, 8))
@pytest.mark.parametrize("shape", GEMV_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("fmt", GEMV_FORMATS, ids=lambda f: f"int{f[0]}-g{f[1]}-{'sym' if f[2] else 'asym'}-{f[3][:3]}")
def test_reference_gate_matrix(fmt, shape, m):
    run_case(*shape, *fmt, m)


@pytest.mark.parametrize("m", (1, 2, 3, 8))
def test_int2_g64_ragged_lane_loop(m):
    # 3072 / 64 = 48 groups: not a whole number of the kernel's steps per warp.
    run_case(3072, 3072, 2, 64, True, "sequential", m)


VALID = [(b, g) for b in (2, 4, 8) for g in (16, 32, 64, 128, 256, None)
         if g is None or g % (128 // b) == 0]


@pytest.mark.parametrize("m", (1, 5, 8))
@pytest.mark.parametrize("layout", ("sequential", "interleaved"))
@pytest.mark.parametrize("sym", (True, False), ids=("sym", "asym"))
@pytest.mark.parametrize("bits,gs", VALID, ids=lambda v: str(v))
def test_every_format_small(bits, gs, sym, layout, m):
    run_case(64, 512, bits, gs, sym, layout, m, seed=1)


@pytest.mark.parametrize("n,k", [(1, 512), (7, 256), (37, 1024), (100, 768), (149, 640),
                                 (300, 4224), (1000, 128)])
@pytest.mark.parametrize("bits,gs", [(4, 128), (2, 64), (8, None), (4, 32), (8, 16)])
def test_ragged_shapes(n, k, bits, gs):
    if gs is not None and k % gs:
        pytest.skip("K not a multiple of the group")
    for m in (1, 8):
        run_case(n, k, bits, gs, False, "sequential", m, seed=n + k)


BENCH = [(8, None, True), (4, 128, False), (2, 64, False)]


# Activations too large for one CTA's shared memory (M x K x 2 > 100 KB) are
# split along K over a cluster of 2, 4 or 8 CTAs that combine their partial
# sums through distributed shared memory.
SPLIT_K = [
    (1000, 11008, 4, 128, False, 8),   # 2 CTAs per cluster
    (333, 11008, 2, 64, False, 8),
    (517, 11008, 8, None, True, 8),    # per-channel
    (257, 11008, 8, None, False, 6),   # per-channel, asymmetric
    (1000, 12288, 4, 128, True, 5),
    (300, 16384, 4, 64, False, 8),     # 4 CTAs
    (200, 28672, 4, 128, False, 8),    # 8 CTAs
    (129, 28672, 2, 64, True, 7),
    (64, 24576, 8, 128, False, 8),
]


@pytest.mark.parametrize("n,k,bits,gs,sym,m", SPLIT_K,
                         ids=lambda v: str(v))
def test_split_k_clusters(n, k, bits, gs, sym, m):
    run_case(n, k, bits, gs, sym, "sequential", m, seed=n + k + m)
    run_case(n, k, bits, gs, sym, "interleaved", m, seed=n + k + m + 1)


@pytest.mark.parametrize("m", (1, 4, 8))
@pytest.mark.parametrize("n,k", [(4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("fmt", BENCH, ids=("int8-perch-sym", "int4-g128-asym", "int2-g64-asym"))
def test_bitwidth_sweep_configs(fmt, n, k, m):
    """The benchmark's bit-width sweep at full size."""
    run_case(n, k, *fmt, "sequential", m, seed=7)


@pytest.mark.parametrize("case", load_golden("known_answers.json")["cases"],
                         ids=lambda c: f"{c['N']}x{c['K']}-int{c['bits']}")
def test_against_reference_recorded_outputs(case):
    """The reference's own F.linear outputs at the benchmark shapes."""
    w, x = bench_inputs(case["N"], case["K"])
    qw, s, z = pack_np(w.numpy(), case["bits"], case["group_size"], case["symmetric"], "sequential")
    y = gpu_gemv(x.numpy(), qw, s, z, case["bits"], case["group_size"] or case["K"],
                 case["symmetric"], "sequential")
    yref = fp16_from_hex(case["y_fp16_hex"], (1, case["N"]))
    assert P.max_rel_err(y, yref) <= REL_TOL


@pytest.mark.parametrize("n,k", [(4096, 4096), (12288, 4096), (4096, 14336), (28672, 8192),
                                 (8192, 28672), (128256, 4096)])
def test_shape_sweep_configs(n, k):
    """BASELINE config 3 (INT4 g128 asym, M=1) at full size. Packed on the GPU
    by the product packer (bit-exact with the reference, see test_packer), then
    checked against the C oracle on the same packed tensors."""
    torch.manual_seed(0)
    w = torch.randn(n, k, dtype=torch.float16, device="cuda") * 0.02
    x = torch.randn(1, k, dtype=torch.float16, device="cuda")
    pw = quantize_tensor(w, QuantConfig(4, 128, False))
    del w
    y = dequant_cuda.gemv(x, pw.qweight, pw.scales, pw.zeros, 4, 128, False, False)
    qw, s, z = pw.qweight.cpu().numpy(), pw.scales.cpu().numpy(), pw.zeros.cpu().numpy()
    check_against_oracle(x.cpu().numpy(), qw, s, z, 4, 128, False, "sequential", y.cpu().numpy(),
                         exact_criterion=n * k <= 64 * 2 ** 20)


@pytest.mark.parametrize("bits", (2, 4, 8))
@pytest.mark.parametrize("zkind", ("skew", "large", "negative", "fractional", "mixed"))
def test_zero_point_edge_cases(bits, zkind):
    """Zero-points outside [-1024, 1024] or non-integer take the exact fp32
    residual path; results must still meet both criteria."""
    n, k, gs = 96, 1024, 128 if bits != 2 else 64
    rng = np.random.default_rng(bits * 10 + len(zkind))
    x = torch.randn(8, k, dtype=torch.float16, generator=torch.Generator().manual_seed(3)).numpy()
    if zkind == "skew":
        w = (rng.random((n, k)) * 0.5 + 2.0).astype(np.float16)
        qw, s, z = pack_np(w, bits, gs, False, "sequential")
    else:
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
        qw, s, z = pack_np(w, bits, gs, False, "sequential")
        z = z.astype(np.float32)
        if zkind == "large":
            z = z + 1500.0
        elif zkind == "negative":
            z = z - 3000.0
        elif zkind == "fractional":
            z = z + 0.5
        else:
            z = z + rng.choice([0.0, 2000.0, -1500.25, 0.75], size=z.shape)
        z = z.astype(np.float16)
        s = (s.astype(np.float32) * 0.01).astype(np.float16)  # keep |W| moderate
    for m in (1, 8):
        y = gpu_gemv(x[:m], qw, s, z, bits, gs, False, "sequential")
        check_against_oracle(x[:m], qw, s, z, bits, gs, False, "sequential", y)


@pytest.mark.parametrize("bits,gs", [(4, 128), (2, 64), (8, None)])
def test_unaligned_metadata_takes_the_plain_load_path(bits, gs):
    """Scales/zeros that are only 2-byte aligned cannot be bulk-copied; the
    general kernel then reads them from global memory. Both paths meet both
    criteria."""
    torch.manual_seed(11)
    n, k = 1000, 2048
    w = (torch.randn(n, k, dtype=torch.float16) * 0.02).numpy()
    x = torch.randn(4, k, dtype=torch.float16).numpy()
    qw, s, z = pack_np(w, bits, gs, False, "sequential")
    xd, qd, sd, zd = to_dev(x, qw, s, z)
    y_aligned = dequant_cuda.gemv(xd, qd, sd, zd, bits, gs or k, False, False)
    # Same values at an address that is 2 mod 16.
    s_buf = torch.empty(sd.numel() + 1, dtype=torch.float16, device="cuda")
    z_buf = torch.empty(zd.numel() + 1, dtype=torch.float16, device="cuda")
    s_off = s_buf[1:].view(sd.shape)
    z_off = z_buf[1:].view(zd.shape)
    s_off.copy_(sd)
    z_off.copy_(zd)
    assert s_off.data_ptr() % 16 == 2
    y_off = dequant_cuda.gemv(xd, qd, s_off, z_off, bits, gs or k, False, False)
    check_against_oracle(x, qw, s, z, bits, gs, False, "sequential", y_aligned.cpu().numpy())
    check_against_oracle(x, qw, s, z, bits, gs, False, "sequential", y_off.cpu().numpy())


def test_rejections():
    """INT2 g32 and M=9 raise RuntimeError (scripts/test_dequant_kernel.py:174-191)."""
    dev = "cuda"
    pw = quantize_tensor(torch.randn(64, 256, dtype=torch.float16, device=dev),
                         QuantConfig(2, 32, True))
    x = torch.randn(1, 256, dtype=torch.float16, device=dev)
    with pytest.raises(RuntimeError, match="INT2 with group_size 32"):
        dequant_cuda.gemv(x, pw.qweight, pw.scales, pw.zeros, 2, 32, True, False)
    pw = quantize_tensor(torch.randn(64, 256, dtype=torch.float16, device=dev),
                         QuantConfig(4, 128, True))
    x9 = torch.randn(9, 256, dtype=torch.float16, device=dev)
    with pytest.raises(RuntimeError, match="M=9"):
        dequant_cuda.gemv(x9, pw.qweight, pw.scales, pw.zeros, 4, 128, True, False)
    xs = torch.randn(1, 257, dtype=torch.float16, device=dev)[:, 1:]
    with pytest.raises(RuntimeError):
        dequant_cuda.gemv(xs, pw.qweight, pw.scales, pw.zeros, 4, 128, True, False)


def test_negative_control_single_flipped_bit():
    """One flipped code bit must break the criterion at [0, 0] and nowhere else
    (scripts/test_dequant_kernel.py:194-217)."""
    torch.manual_seed(0)
    n = k = 3072
    w = (torch.randn(n, k, dtype=torch.float16) * 0.02).numpy()
    qw, s, z = pack_np(w, 4, 128, True, "sequential")
    x = torch.zeros(1, k, dtype=torch.float16)
    x.normal_()
    x[0, 0] = 1.0
    x = x.numpy()
    we = P.exact_weight(qw, s, z, 4, 128, True, "sequential", k).astype(np.float64)
    ref = x.astype(np.float64) @ we.T
    bad = qw.copy()
    bad[0, 0] ^= 1
    y = gpu_gemv(x, bad, s, z, 4, 128, True, "sequential")
    err, tol = P.gemv_criterion(y, ref, np.abs(we), np.abs(x.astype(np.float64)))
    assert err[0, 0] > tol[0, 0]
    assert int((err > tol).sum()) == 1


def test_batch_rows_are_independent_and_deterministic():
    """Size-independent properties at a full benchmark shape: repeated calls
    are bit-identical; an output row does not depend on the other activation
    rows of the batch (bit for bit, same M); and it matches the M=1 call on
    that activation row to within fp32 summation order."""
    torch.manual_seed(5)
    w = torch.randn(11008, 4096, dtype=torch.float16, device="cuda") * 0.02
    for bits, gs, sym in BENCH:
        pw = quantize_tensor(w, QuantConfig(bits, gs, sym))
        x = torch.randn(8, 4096, dtype=torch.float16, device="cuda")
        args = (pw.qweight, pw.scales, pw.zeros, bits, gs or 4096, sym, False)
        y8 = dequant_cuda.gemv(x, *args)
        assert torch.equal(y8, dequant_cuda.gemv(x, *args))
        x_other = torch.randn(8, 4096, dtype=torch.float16, device="cuda")
        for m in range(8):
            mixed = x_other.clone()
            mixed[m] = x[m]
            assert torch.equal(dequant_cuda.gemv(mixed, *args)[m], y8[m])
            y1 = dequant_cuda.gemv(x[m:m + 1].contiguous(), *args)[0].float()
            d = (y1 - y8[m].float()).abs().max().item()
            assert d <= 1e-3 * y8[m].float().abs().max().item()


def test_graph_capture_replays_live_input():
    """scripts/test_dequant_kernel.py:220-252."""
    torch.manual_seed(0)
    n = k = 3072
    w = torch.randn(n, k, dtype=torch.float16, device="cuda") * 0.02
    pw = quantize_tensor(w, QuantConfig(4, 128, False))
    args = (pw.qweight, pw.scales, pw.zeros, 4, 128, False, False)
    x = torch.randn(1, k, dtype=torch.float16, device="cuda")
    x2 = torch.randn(1, k, dtype=torch.float16, device="cuda")
    eager1 = dequant_cuda.gemv(x, *args).clone()
    eager2 = dequant_cuda.gemv(x2, *args).clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            dequant_cuda.gemv(x, *args)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = dequant_cuda.gemv(x, *args)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager1)
    x.copy_(x2)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager2)


@pytest.fixture
def streaming_only():
    """dqg_gemv restricted to the streaming (and general) kernels."""
    lib = _native.lib()
    prev = lib.dqg_set_gemv_path(1)
    yield
    lib.dqg_set_gemv_path(prev)


@pytest.mark.parametrize("m", (1, 3, 8))
@pytest.mark.parametrize("n,k", [(4096, 11008), (11008, 4096), (3072, 3072), (149, 640)])
@pytest.mark.parametrize("fmt", [(4, 128, False), (2, 64, False), (4, 128, True), (8, 64, False)],
                         ids=("int4-g128-asym", "int2-g64-asym", "int4-g128-sym", "int8-g64-asym"))
def test_streaming_kernel_on_direct_shapes(streaming_only, fmt, n, k, m):
    """Shapes the direct kernel takes by default, through the streaming
    kernel: it stays correct for every caller that forces it."""
    run_case(n, k, *fmt, "sequential", m, seed=n + m)


@pytest.fixture
def direct_everywhere():
    """dqg_gemv takes the direct kernel wherever it applies, at any M."""
    lib = _native.lib()
    prev = lib.dqg_set_gemv_path(2)
    yield
    lib.dqg_set_gemv_path(prev)


@pytest.mark.parametrize("m", (1, 2, 4, 8))
@pytest.mark.parametrize("fmt", [(4, 128, False), (4, 64, True), (8, 64, False), (4, 32, False),
                                 (8, 32, True)],
                         ids=lambda f: f"int{f[0]}-g{f[1]}-{'sym' if f[2] else 'asym'}")
def test_direct_kernel_formats(direct_everywhere, fmt, m):
    """Every 4/8-bit group size whose group is one tensor-core step of a lane
    (the direct kernel's domain), at every activation-row count, interleaved
    and sequential, ragged rows and a group count that is not a whole number
    of units."""
    bits, gs, sym = fmt
    for n, k in ((1000, 43 * gs), (37, 11 * gs), (4096, 4096)):
        run_case(n, k, bits, gs, sym, "sequential", m, seed=n + m)
        run_case(n, k, bits, gs, sym, "interleaved", m, seed=n + m + 1)


def test_no_kernel_gave_up_a_wait():
    torch.cuda.synchronize()
    assert _native.device_status(torch.cuda.current_device()) == 0
