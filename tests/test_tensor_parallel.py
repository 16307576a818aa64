"""Tensor-parallel sharding of packed linear layers.

CPU tests (gloo, world size 2) cover the host logic: balanced uneven splits on
group boundaries (the 11008 = 86 x 128 rule), bit-exact shards, the
column-parallel gather and the row-parallel all-reduce (with a CPU stand-in
for the GEMV: the reference CPU path x @ packer.dequantize(shard)^T), and a
rank that fails before the collective (the survivor gets an error, no hang).
The GPU test runs two NCCL ranks with the real kernel when two GPUs exist.
"""

from __future__ import annotations

import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from dequant_project_b200.packer import QuantConfig, dequantize, quantize_tensor
from dequant_project_b200.tensor_parallel import (intermediate_bounds, shard_columns,
                                                  shard_rows, split_bounds)

FORMATS = [(4, 128, False), (4, 128, True), (2, 64, False), (8, None, True), (8, None, False),
           (4, None, False)]


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_split_bounds_balanced():
    for units in (1, 7, 86, 224, 4096):
        for world in (1, 2, 3, 4, 8):
            if units < world:
                with pytest.raises(ValueError):
                    split_bounds(units, world)
                continue
            b = split_bounds(units, world)
            sizes = [hi - lo for lo, hi in zip(b[:-1], b[1:])]
            assert b[0] == 0 and b[-1] == units and len(b) == world + 1
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)


def test_llama7b_intermediate_split_on_groups():
    """11008 = 86 groups of 128: 8 ranks get 11,11,11,11,11,11,10,10 groups."""
    b = intermediate_bounds(11008, QuantConfig(4, 128, False), 8)
    assert [(hi - lo) // 128 for lo, hi in zip(b[:-1], b[1:])] == [11] * 6 + [10] * 2
    assert all(x % 128 == 0 for x in b) and b[-1] == 11008


@pytest.mark.parametrize("bits,gs,sym", FORMATS)
@pytest.mark.parametrize("world", (2, 3, 8))
def test_shards_are_bit_exact_slices(bits, gs, sym, world):
    torch.manual_seed(world)
    n, k = 72, 1024
    pw = quantize_tensor(torch.randn(n, k, dtype=torch.float16) * 0.02, QuantConfig(bits, gs, sym))
    full = dequantize(pw)
    cols = [shard_columns(pw, world, r) for r in range(world)]
    assert torch.equal(torch.cat([c.qweight for c in cols]), pw.qweight)
    assert torch.equal(torch.cat([dequantize(c) for c in cols]), full)
    rows = [shard_rows(pw, world, r) for r in range(world)]
    assert [lo for _, lo, _ in rows] + [rows[-1][2]] == sorted({lo for _, lo, _ in rows} | {k})
    for shard, lo, hi in rows:
        assert shard.shape == (n, hi - lo)
        assert torch.equal(dequantize(shard), full[:, lo:hi])


def test_row_shard_rejects_misaligned_bounds():
    pw = quantize_tensor(torch.randn(16, 512, dtype=torch.float16), QuantConfig(4, 128, False))
    with pytest.raises(ValueError, match="multiples of 128"):
        shard_rows(pw, 2, 0, bounds=[0, 200, 512])


def _run_ranks(target, world, args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    t0 = time.time()
    while len(out) < world and time.time() - t0 < timeout:
        try:
            r, status, a, b = q.get(timeout=1)
            out[r] = (status, a, b)
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("cfg", [(4, 128, False), (8, None, True), (2, 64, False)])
def test_gloo_two_ranks_match_single_process(cfg):
    import tp_workers

    n, k, m = 200, 1152, 3   # 9 groups of 128 (uneven K split), 200 rows
    out = _run_ranks(tp_workers.tp_forward, 2, (free_port(), "gloo", n, k, cfg, m))
    assert set(out) == {0, 1}, out
    for r, (status, a, _) in out.items():
        assert status == "ok", a
    # Single-process reference: the same packed weight, the same CPU stand-in.
    pw, x, bias = tp_workers._layer_inputs(n, k, cfg, m, torch.device("cpu"))
    ref = (tp_workers._cpu_linear(x, pw).float() + bias.float())
    y_col, y_row = out[0][1], out[0][2]
    # Column-parallel: each output row is computed exactly as without TP.
    assert torch.equal(y_col, (tp_workers._cpu_linear(x, pw) + bias))
    assert torch.equal(out[1][1], y_col) and torch.equal(out[1][2], y_row)
    # Row-parallel: fp16 partials summed by the all-reduce.
    rel = ((y_row.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= 2e-3


def test_rank_failure_surfaces_as_error_not_hang():
    import tp_workers

    t0 = time.time()
    out = _run_ranks(tp_workers.tp_rank_fails, 2, (free_port(),), timeout=90)
    assert out.get(1, ("missing",))[0] == "error"
    assert out.get(0, ("missing",))[0] == "error", out.get(0)
    assert time.time() - t0 < 90


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_nccl_two_gpus_match_one_gpu():
    import tp_workers

    from dequant_project_b200 import quant_linear

    n, k, m, cfg = 4096, 11008, 1, (4, 128, False)
    out = _run_ranks(tp_workers.tp_forward, 2, (free_port(), "nccl", n, k, cfg, m), timeout=300)
    assert set(out) == {0, 1}, out
    for r, (status, a, _) in out.items():
        assert status == "ok", a
    pw, x, bias = tp_workers._layer_inputs(n, k, cfg, m, torch.device("cuda", 0))
    ref = (quant_linear.gemv(x, pw).float() + bias.float()).cpu()
    y_col, y_row = out[0][1], out[0][2]
    assert torch.equal(y_col.float(), ref) or \
        ((y_col.float() - ref).abs().max() / ref.abs().max()).item() <= 2e-3
    assert ((y_row.float() - ref).abs().max() / ref.abs().max()).item() <= 2e-3
