"""Decoder step on the GPU: the element-wise kernels against torch's formulas,
the packed-GEMV decoder against the same decoder with dequantize-then-matmul
linears, CUDA-graph replay against eager, and two NCCL ranks against one GPU.
"""

from __future__ import annotations

import socket
import time

import pytest
import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

from decoder_reference import max_rel_err, reference_step  # noqa: E402
from dequant_project_b200 import decode_ops  # noqa: E402
from dequant_project_b200.decoder import DecodeGraph, DecoderConfig, TPDecoder  # noqa: E402
from dequant_project_b200.packer import QuantConfig  # noqa: E402

SMALL = DecoderConfig(n_layers=2, hidden=1024, n_heads=8, n_kv_heads=4, intermediate=2816,
                      vocab=5000)
FORMATS = [(4, 128, False), (2, 64, False), (8, None, True)]


def dequant_linear(x, pw):
    from dequant_project_b200.quant_linear import dequantize_cuda
    return (x.float() @ dequantize_cuda(pw).float().t()).to(torch.float16)


def test_add_rms_norm_matches_torch():
    g = torch.Generator(device="cuda").manual_seed(0)
    m, hd = 3, 4096
    h = torch.randn(m, hd, generator=g, device="cuda").half()
    delta = torch.randn(m, hd, generator=g, device="cuda").half()
    w = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")).half()
    h_ref = h + delta
    hf = h_ref.float()
    y_ref = ((hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)) * w.float()).half()
    y = decode_ops.add_rms_norm(h, delta, w, 1e-5)
    assert torch.equal(h, h_ref)                       # the residual add is one fp16 rounding
    torch.testing.assert_close(y, y_ref, rtol=2e-3, atol=1e-3)
    y2 = decode_ops.add_rms_norm(h, None, w, 1e-5)     # no residual: h unchanged
    assert torch.equal(h, h_ref)
    torch.testing.assert_close(y2, y_ref, rtol=2e-3, atol=1e-3)


def test_rope_kv_append_matches_torch_formula():
    g = torch.Generator(device="cuda").manual_seed(1)
    m, hq, hkv, d, cap, pos = 2, 8, 2, 128, 40, 33
    qkv = torch.randn(m, (hq + 2 * hkv) * d, generator=g, device="cuda").half()
    ang = torch.rand(d // 2, generator=g, device="cuda") * 30
    cos = torch.cat([ang.cos(), ang.cos()]).float()
    sin = torch.cat([ang.sin(), ang.sin()]).float()
    kc = torch.randn(m, hkv, cap, d, generator=g, device="cuda").half()
    vc = torch.randn(m, hkv, cap, d, generator=g, device="cuda").half()
    kc0, vc0 = kc.clone(), vc.clone()

    def rot(t):
        tf = t.float()
        r = torch.cat([-tf[..., d // 2:], tf[..., :d // 2]], dim=-1)
        return (tf * cos + r * sin).half()

    q = decode_ops.rope_kv_append(qkv, cos, sin, kc, vc, pos, hq, hkv)
    nq, nkv = hq * d, hkv * d
    assert torch.equal(q, rot(qkv[:, :nq].reshape(m, hq, d)))
    assert torch.equal(kc[:, :, pos], rot(qkv[:, nq:nq + nkv].reshape(m, hkv, d)))
    assert torch.equal(vc[:, :, pos], qkv[:, nq + nkv:].reshape(m, hkv, d))
    others = [t for t in range(cap) if t != pos]
    assert torch.equal(kc[:, :, others], kc0[:, :, others])
    assert torch.equal(vc[:, :, others], vc0[:, :, others])


def test_silu_mul_matches_torch():
    g = torch.Generator(device="cuda").manual_seed(2)
    gu = (3 * torch.randn(5, 2 * 2816, generator=g, device="cuda")).half()
    ref = (F.silu(gu[:, :2816].float()) * gu[:, 2816:].float()).half()
    torch.testing.assert_close(decode_ops.silu_mul(gu), ref, rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("batch", (1, 8))
def test_decoder_matches_dequantized_reference(fmt, batch):
    bits, gs, sym = fmt
    q = QuantConfig(bits, gs, sym)
    dec = TPDecoder(SMALL, q, device="cuda", seed=5, batch=batch, kv_len=100)
    ref = TPDecoder(SMALL, q, device="cuda", seed=5, batch=batch, kv_len=100,
                    linear_fn=dequant_linear)
    tokens = torch.arange(batch, device="cuda") * 611 % SMALL.vocab
    a = dec.step(tokens, 100).float()
    b = ref.step(tokens, 100).float()
    err = ((a - b).abs().max() / b.abs().max()).item()
    assert err < 1e-2, err


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("batch", (1, 8))
def test_decoder_matches_fp32_restatement(fmt, batch):
    """The GPU step (fused GEMVs, element-wise kernels, attention) against the
    independent per-head fp32 restatement that rounds to fp16 where the
    decoder stores fp16: within north_star's 2e-3 on the logits."""
    dec = TPDecoder(SMALL, QuantConfig(*fmt), device="cuda", seed=5, batch=batch, kv_len=100)
    tokens = torch.arange(batch, device="cuda") * 611 % SMALL.vocab
    ref = reference_step(dec, tokens, 100, storage=torch.float16)
    out = dec.step(tokens, 100)
    assert max_rel_err(out, ref) < 2e-3


def test_graph_replay_matches_eager():
    dec = TPDecoder(SMALL, QuantConfig(4, 128, False), device="cuda", seed=6, batch=1,
                    kv_len=64)
    tokens = torch.tensor([17], device="cuda")
    eager = dec.step(tokens, 64).clone()
    gr = DecodeGraph(dec, 64)
    gr.tokens.copy_(tokens)
    out = gr.replay().clone()
    torch.cuda.synchronize()
    gr.release()
    assert torch.equal(out, eager)


@pytest.mark.parametrize("fmt", [(4, 128, False), (8, 64, True), (4, 64, False)])
@pytest.mark.parametrize("m", [1, 2, 8])
def test_gemv_swiglu_matches_gemv_then_silu(fmt, m):
    """The gate/up GEMV fused with SwiGLU (rows interleaved by eights) against
    the GEMV of the same interleaved weight, de-interleaved, then silu_mul."""
    from dequant_project_b200 import dequant_cuda
    from dequant_project_b200.packer import PackedWeight, quantize_tensor
    bits, gs, sym = fmt
    ir, k = 2816, 1024
    g = torch.Generator(device="cuda").manual_seed(m * 31 + bits)
    w = torch.randn(2 * ir, k, generator=g, device="cuda").half() * 0.05
    pw = quantize_tensor(w, QuantConfig(bits, gs, sym))
    order = decode_ops.gate_up_order(ir).cuda()
    il = PackedWeight(pw.qweight[order].contiguous(), pw.scales[order].contiguous(),
                      None if pw.zeros is None else pw.zeros[order].contiguous(), pw.config,
                      pw.shape)
    x = torch.randn(m, k, generator=g, device="cuda").half()
    assert decode_ops.gemv_swiglu_supported(m, 2 * ir, k, bits, gs)
    for _ in range(2):
        act = decode_ops.gemv_swiglu(x, il)
        y = dequant_cuda.gemv(x, il.qweight, il.scales, il.zeros, bits, gs, sym, False)
        ref = decode_ops.silu_mul(y[:, torch.argsort(order)].contiguous())
        assert act.shape == (m, ir)
        torch.testing.assert_close(act.float(), ref.float(), rtol=2e-3,
                                   atol=2e-3 * ref.float().abs().max().item())
        assert (act == ref).float().mean().item() > 0.99   # most outputs bit-identical


def test_gemv_swiglu_rejects_shapes_without_a_plan():
    from dequant_project_b200 import _native
    assert not decode_ops.gemv_swiglu_supported(1, 2 * 2816, 11008, 4, 128)   # K > 6144
    assert not decode_ops.gemv_swiglu_supported(1, 2 * 2816, 4096, 2, 64)     # 2-bit codes
    assert not decode_ops.gemv_swiglu_supported(1, 2 * 2816 + 8, 4096, 4, 128)   # N % 16
    q = torch.zeros(16, 11008 // 8, dtype=torch.int32, device="cuda")
    s = torch.ones(16, 86, dtype=torch.float16, device="cuda")
    x = torch.zeros(1, 11008, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 8, dtype=torch.float16, device="cuda")
    rc = _native.lib().dqg_gemv_swiglu(x.data_ptr(), q.data_ptr(), s.data_ptr(), None,
                                       out.data_ptr(), 1, 16, 11008, 4, 128, 1, 0,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 2 and b"no direct-kernel plan" in _native.lib().dqg_last_error()


def test_decoder_swiglu_fusion_matches_separate_kernels():
    q = QuantConfig(4, 128, False)
    a = TPDecoder(SMALL, q, device="cuda", seed=8, batch=2, kv_len=64)
    b = TPDecoder(SMALL, q, device="cuda", seed=8, batch=2, kv_len=64, fuse_swiglu=False)
    assert a.gu_order is not None and b.gu_order is None
    tokens = torch.tensor([5, 77], device="cuda")
    assert max_rel_err(a.step(tokens, 64), b.step(tokens, 64).float()) < 2e-3


def test_l2_prefetch_changes_nothing_but_timing():
    """The decoder with its element-wise ops prefetching later weights into
    L2 gives bit-identical logits, eager and graph-replayed, to the one
    without."""
    q = QuantConfig(4, 128, False)
    a = TPDecoder(SMALL, q, device="cuda", seed=7, batch=2, kv_len=64, l2_prefetch=True)
    b = TPDecoder(SMALL, q, device="cuda", seed=7, batch=2, kv_len=64)
    assert a._pf is not None and b._pf is None
    plan = a.prefetch_plan()
    assert plan[(0, "norm1")] == [(0, "qkv")] and plan[(1, "rope")] == [(1, "o"), (1, "gu")]
    assert (1, "silu") not in plan           # nothing after the last layer's down projection
    tokens = torch.tensor([17, 4001], device="cuda")
    assert torch.equal(a.step(tokens, 64), b.step(tokens, 64))
    gr = DecodeGraph(a, 64)
    gr.tokens.copy_(tokens)
    out = gr.replay().clone()
    torch.cuda.synchronize()
    gr.release()
    assert torch.equal(out, b.step(tokens, 64))


def test_prefetch_ranges_are_checked():
    """Prefetch ranges go through the C ABI's checks: more than 8, a range
    that runs past its device allocation and a host pointer are rejected; unaligned
    starts and odd sizes are trimmed, and the op's output does not change."""
    from dequant_project_b200 import _native
    m, hd = 1, 1024
    h = torch.randn(m, hd, device="cuda").half()
    w = torch.ones(hd, device="cuda").half()
    buf = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    ref = decode_ops.add_rms_norm(h, None, w, 1e-5)
    ok = _native.L2Spans.of([(buf.data_ptr() + 3, 5000), (buf.data_ptr(), buf.numel())])
    assert torch.equal(decode_ops.add_rms_norm(h, None, w, 1e-5, ok), ref)
    assert torch.equal(decode_ops.silu_mul(torch.cat([h, h], 1), ok),
                       decode_ops.silu_mul(torch.cat([h, h], 1)))
    with pytest.raises(ValueError):
        _native.L2Spans.of([(buf.data_ptr(), 16)] * 9)
    # Past the end of the device allocation that holds buf (the caching
    # allocator's segment, which may be larger than buf itself).
    bad = _native.L2Spans.of([(buf.data_ptr(), 1 << 40)])
    with pytest.raises(RuntimeError, match="past the end"):
        decode_ops.add_rms_norm(h, None, w, 1e-5, bad)
    host = torch.empty(4096, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="prefetch range"):
        decode_ops.add_rms_norm(h, None, w, 1e-5, _native.L2Spans.of([(host.data_ptr(), 4096)]))
    over = _native.L2Spans.of([(buf.data_ptr(), 16)])
    over.n = 9
    with pytest.raises(RuntimeError, match="prefetch.n"):
        decode_ops.add_rms_norm(h, None, w, 1e-5, over)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_two_ranks_match_one_gpu():
    import tp_workers
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_workers.decoder_step_nccl, args=(r, 2, port, q))
             for r in range(2)]
    for p in procs:
        p.start()
    out, t0 = {}, time.time()
    while len(out) < 2 and time.time() - t0 < 300:
        try:
            r, status, val = q.get(timeout=1)
            out[r] = (status, val)
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert set(out) == {0, 1}, out
    for r, (status, val) in out.items():
        assert status == "ok", val
    one = TPDecoder(SMALL, QuantConfig(4, 128, False), device="cuda", seed=5, batch=2,
                    kv_len=100)
    ref = one.step(torch.tensor([3, 4001], device="cuda"), 100).float().cpu()
    for r in (0, 1):
        err = ((out[r][1].float() - ref).abs().max() / ref.abs().max()).item()
        assert err < 5e-3, err
