"""Tensor-parallel decoder step: host logic on the CPU.

The decoder's linear layers run through a CPU stand-in for the GEMV (the
reference CPU path, x @ packer.dequantize(W)^T in fp32, fp16 out) and its
element-wise steps through the torch formulas of ``decode_ops``. Checked here:
the single-rank step against an independent fp32 restatement of a Llama decode
step (loops over heads, no fused steps), two gloo ranks against one rank
(head split, intermediate split on group boundaries, the two all-reduces per
layer, the vocabulary all-gather), and the argument checks.
"""

from __future__ import annotations

import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from decoder_reference import max_rel_err, reference_step
from dequant_project_b200.decoder import DecoderConfig, TPDecoder, cat_rows
from dequant_project_b200.packer import QuantConfig, dequantize, quantize_tensor

TINY = DecoderConfig(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, intermediate=640,
                     vocab=1000)
QCFG = QuantConfig(4, 64, False)


def cpu_linear(x, pw):
    w = dequantize(pw).float()
    return (x.float() @ w.t()).to(torch.float16)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_single_rank_matches_fp32_reference():
    dec = TPDecoder(TINY, QCFG, seed=3, batch=2, kv_len=24, linear_fn=cpu_linear)
    tokens = torch.tensor([5, 977])
    pos = dec.kv_len
    ref = reference_step(dec, tokens, pos)        # reads the cache before the step writes it
    ref16 = reference_step(dec, tokens, pos, storage=torch.float16)
    logits = dec.step(tokens, pos).float()
    assert max_rel_err(logits, ref) < 1e-2
    assert max_rel_err(logits, ref16) < 2e-3


def test_step_writes_cache_slot_and_is_repeatable():
    dec = TPDecoder(TINY, QCFG, seed=1, batch=1, kv_len=8, max_new=2, linear_fn=cpu_linear)
    before = [c.clone() for c in dec.k_cache]
    tok = torch.tensor([7])
    a = dec.step(tok, 8)
    for layer, c in enumerate(dec.k_cache):
        assert torch.equal(c[:, :, :8], before[layer][:, :, :8])
        assert c[:, :, 8].abs().sum() > 0 and torch.equal(c[:, :, 9], before[layer][:, :, 9])
    assert torch.equal(dec.step(tok, 8), a)       # same slot rewritten with the same values
    with pytest.raises(ValueError, match="outside the cache"):
        dec.step(tok, 10)


def test_cat_rows_is_row_concatenation():
    torch.manual_seed(0)
    parts = [quantize_tensor(torch.randn(n, 256, dtype=torch.float16) * 0.02, QCFG)
             for n in (64, 32, 96)]
    cat = cat_rows(parts)
    assert cat.shape == (192, 256)
    assert torch.equal(dequantize(cat), torch.cat([dequantize(p) for p in parts]))
    with pytest.raises(ValueError):
        cat_rows([parts[0], quantize_tensor(torch.randn(8, 128, dtype=torch.float16), QCFG)])


def test_rejects_head_counts_that_do_not_split():
    with pytest.raises(ValueError, match="do not split"):
        TPDecoder(TINY, QCFG, world=3, linear_fn=cpu_linear)


def run_gloo_decoder(world, fmt, cfg_kw=None, batch=2, kv_len=24, tokens=(5, 977),
                     limit_s=300):
    """Spawn ``world`` gloo ranks of tp_workers.decoder_step; returns their
    logits by rank (asserting every rank succeeded)."""
    import tp_workers
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=tp_workers.decoder_step,
                         args=(r, world, port, q, fmt, cfg_kw, batch, kv_len, tokens))
             for r in range(world)]
    for p in procs:
        p.start()
    out, t0 = {}, time.time()
    while len(out) < world and time.time() - t0 < limit_s:
        try:
            r, status, val = q.get(timeout=1)
            out[r] = (status, val)
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert set(out) == set(range(world)), out
    for r, (status, val) in out.items():
        assert status == "ok", val
    return {r: val for r, (_, val) in out.items()}


@pytest.mark.parametrize("fmt", [(4, 64, False), (8, None, True), (2, 64, False)],
                         ids=("int4-g64", "int8-perchannel", "int2-g64"))
def test_gloo_two_ranks_match_one_rank(fmt):
    out = run_gloo_decoder(2, fmt)
    assert torch.equal(out[0], out[1])
    one = TPDecoder(TINY, QuantConfig(*fmt), seed=3, batch=2, kv_len=24, linear_fn=cpu_linear)
    ref = one.step(torch.tensor([5, 977]), one.kv_len).float()
    assert max_rel_err(out[0], ref) < 5e-3


# Llama-2-7B-shaped (multi-head attention, 11008 = 86 groups of 128 split 11/10
# over 8 ranks -> here 43 groups of 64 split 6/5) and Llama-3-70B-shaped
# (grouped KV heads, one KV head per rank at width 8) small decoders; uneven
# vocabulary split.
WIDE_MHA = dict(n_layers=2, hidden=512, n_heads=16, n_kv_heads=16, intermediate=43 * 64,
                vocab=1003)
WIDE_GQA = dict(n_layers=2, hidden=512, n_heads=16, n_kv_heads=8, intermediate=43 * 64,
                vocab=1003, rope_theta=500000.0)


@pytest.mark.parametrize("world", (4, 8))
@pytest.mark.parametrize("cfg_kw", (WIDE_MHA, WIDE_GQA), ids=("mha-7b-like", "gqa-70b-like"))
def test_gloo_wide_tensor_parallel_matches_one_rank(world, cfg_kw):
    """Every tensor-parallel width the scaling bench runs: heads split several
    per rank (or one KV head per rank), the intermediate split unevenly on
    group boundaries, the vocabulary unevenly; all ranks return the same
    logits, which match the one-rank decoder and the fp32 restatement."""
    fmt = (4, 64, False)
    cfg = DecoderConfig(**cfg_kw)
    from dequant_project_b200.tensor_parallel import intermediate_bounds
    b = intermediate_bounds(cfg.intermediate, QuantConfig(*fmt), world)
    sizes = {b[i + 1] - b[i] for i in range(world)}
    assert len(sizes) == 2, sizes                          # uneven by one group
    out = run_gloo_decoder(world, fmt, cfg_kw, batch=2, kv_len=20, tokens=(11, 1001))
    for r in range(1, world):
        assert torch.equal(out[r], out[0])
    one = TPDecoder(cfg, QuantConfig(*fmt), seed=3, batch=2, kv_len=20, linear_fn=cpu_linear)
    tokens = torch.tensor([11, 1001])
    ref32 = reference_step(one, tokens, 20, storage=torch.float16)
    ref = one.step(tokens, 20).float()
    assert max_rel_err(out[0], ref) < 5e-3
    assert max_rel_err(out[0], ref32) < 5e-3
    assert max_rel_err(ref, ref32) < 5e-3


def test_step_bytes_follow_the_reference_decode_model():
    """Per-rank bytes of a step: the packed weights are exactly the reference
    byte model's quantized bytes (numel * bits / 8 + one fp16 scale and zero
    per group, dequant/byte_model.py:165-176) for the layers and the LM head,
    split without overlap across ranks; the KV term reads positions 0..pos and
    writes one slot."""
    cfg, q = TINY, QCFG
    d = cfg.head_dim
    quantizable = cfg.n_layers * (cfg.hidden * (cfg.n_heads + 2 * cfg.n_kv_heads) * d
                                  + cfg.hidden * cfg.n_heads * d
                                  + 3 * cfg.hidden * cfg.intermediate) + cfg.vocab * cfg.hidden
    expect = quantizable * q.bits // 8 + quantizable // q.group_size * 2 * 2
    one = TPDecoder(cfg, q, batch=2, kv_len=24, linear_fn=cpu_linear)
    by = one.step_bytes(24)
    assert by["weights"] == expect
    assert by["kv_cache"] == cfg.n_layers * 2 * 2 * cfg.n_kv_heads * d * 2 * (25 + 1)
    ranks = [TPDecoder(cfg, q, world=2, rank=r, batch=2, kv_len=24, linear_fn=cpu_linear)
             for r in range(2)]
    assert sum(r.step_bytes(24)["weights"] for r in ranks) == expect
    assert sum(r.step_bytes(24)["kv_cache"] for r in ranks) == by["kv_cache"]


def test_rank_failure_ends_the_step_with_an_error_not_a_hang():
    import tp_workers
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=tp_workers.decoder_rank_fails, args=(r, 2, port, q))
             for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    out = {}
    while len(out) < 2 and time.time() - t0 < 120:
        try:
            r, status, val = q.get(timeout=1)
            out[r] = (status, val)
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert out.get(1, ("missing",))[0] == "error"
    assert out.get(0, ("missing",))[0] == "error", out.get(0)
    assert time.time() - t0 < 120


def test_generate_is_greedy_stepping():
    dec = TPDecoder(TINY, QCFG, seed=2, batch=2, kv_len=10, max_new=4, linear_fn=cpu_linear)
    ids = dec.generate(torch.tensor([3, 400]), 4)
    assert ids.shape == (2, 4) and ids.dtype == torch.int64
    dec.reset_cache(2)                      # same cache contents again
    cur, want = torch.tensor([3, 400]), []
    for t in range(4):
        cur = dec.step(cur, 10 + t).argmax(dim=-1)
        want.append(cur)
    assert torch.equal(ids, torch.stack(want, dim=1))
    with pytest.raises(ValueError, match="exceed the cache"):
        dec.generate(torch.tensor([3, 400]), 5)


def test_gate_up_order_interleaves_by_eights():
    """The row order of the fused gate/up + SwiGLU kernel: 8 gate rows, then
    the same outputs' 8 up rows; a permutation that argsort undoes."""
    from dequant_project_b200 import decode_ops
    ir = 24
    order = decode_ops.gate_up_order(ir)
    assert order.tolist()[:16] == list(range(8)) + list(range(ir, ir + 8))
    assert order.tolist()[16:32] == list(range(8, 16)) + list(range(ir + 8, ir + 16))
    assert sorted(order.tolist()) == list(range(2 * ir))
    y = torch.arange(2 * ir, dtype=torch.float32)[None, :]
    assert torch.equal(y[:, order][:, torch.argsort(order)], y)
    with pytest.raises(ValueError):
        decode_ops.gate_up_order(12)
