"""The one-shot peer all-reduce kernel on the GPU.

On one GPU, one launch at a time: the exchange protocol is exercised with a
second rank's buffer that lives on the same device, and the packets that rank
would have sent are written (or left out) by the test before the launch, so
no kernel ever waits for another kernel. With two GPUs: two NCCL processes, the kernel against the fp32 sum of
both ranks' inputs (bit-exact), eager and replayed from a CUDA graph, and the
decoder with the peer all-reduce against the decoder with NCCL's.
"""

from __future__ import annotations

import ctypes
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from dequant_project_b200 import _native

pytestmark = pytest.mark.gpu


def _buffers(cap, world, dev):
    """A receive buffer: [parity 2][source rank world][cap / 2] packets of
    (int32 data word, int32 epoch)."""
    return torch.zeros(8 * world * cap, dtype=torch.uint8, device=dev)


def _packets(buf, cap, world):
    return buf.view(torch.int32).view(2, world, cap // 2, 2)


def _call(inp, out, n, bufs, ctl, cap, rank, world, wait_ns=0):
    ptrs = (ctypes.c_uint64 * world)(*[b.data_ptr() for b in bufs])
    return _native.lib().dqg_peer_allreduce(
        inp.data_ptr(), out.data_ptr(), n, ptrs, ctl.data_ptr(), cap, rank, world, wait_ns,
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("n", [8, 4096, 4104, 65536])
def test_sums_a_peer_whose_packets_have_arrived(cuda_device, n):
    cap, world = 65536, 2
    mine, peer = _buffers(cap, world, cuda_device), _buffers(cap, world, cuda_device)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(n)
    a = torch.randn(n, generator=g, device=cuda_device).half()
    b = torch.randn(n, generator=g, device=cuda_device).half()
    # The first call has epoch 1: rank 1's packets sit in parity half 1, slot 1
    # of this rank's buffer (as rank 1's stores would have left them).
    pk = _packets(mine, cap, world)
    pk[1, 1, :n // 2, 0] = b.view(torch.int32)
    pk[1, 1, :n // 2, 1] = 1
    out = torch.empty_like(a)
    _native.device_status(cuda_device.index, reset=True)
    _native.check(_call(a, out, n, [mine, peer], ctl, cap, 0, world))
    torch.cuda.synchronize()
    assert torch.equal(out, (a.float() + b.float()).half())
    # This rank's words went to slot 0 of the peer's buffer, flagged with the epoch.
    pp = _packets(peer, cap, world)
    assert torch.equal(pp[1, 0, :n // 2, 0], a.view(torch.int32))
    assert bool((pp[1, 0, :n // 2, 1] == 1).all())
    assert int(pp[0].abs().sum()) == 0 and int(pp[1, 1].abs().sum()) == 0
    assert ctl.tolist() == [1, 0]                 # next call: epoch 2, parity 0
    assert _native.device_status(cuda_device.index) == 0


def test_single_rank_is_a_copy(cuda_device):
    cap = 4096
    mine = _buffers(cap, 1, cuda_device)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    a = torch.randn(cap, device=cuda_device).half()
    out = torch.empty_like(a)
    for _ in range(3):                            # epochs 1, 2, 3: both parity halves
        _native.check(_call(a, out, cap, [mine], ctl, cap, 0, 1))
    torch.cuda.synchronize()
    assert torch.equal(out, a) and ctl.tolist() == [3, 0]


def test_missing_peer_gives_up_and_reports(cuda_device):
    cap, world, n = 8192, 2, 8192
    mine, peer = _buffers(cap, world, cuda_device), _buffers(cap, world, cuda_device)
    # Packets of an older call (epoch 3) must not be taken for this one's.
    pk = _packets(mine, cap, world)
    pk[1, 1, :, 1] = 3
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    a = torch.randn(n, device=cuda_device).half()
    out = torch.full_like(a, 3.0)
    _native.device_status(cuda_device.index, reset=True)
    _native.check(_call(a, out, n, [mine, peer], ctl, cap, 0, world, wait_ns=20_000_000))
    torch.cuda.synchronize()                      # returns: the wait ran out after 20 ms
    assert _native.device_status(cuda_device.index, reset=True) & 1
    assert bool((out == 3.0).all()), "a call whose peer never arrived wrote its output"
    assert ctl.tolist() == [1, 0]                 # the call still counted
    assert _native.device_status(cuda_device.index) == 0


def _norm_call(part, h, w, y, bufs, ctl, cap, rank, world, wait_ns=0, eps=1e-5):
    ptrs = (ctypes.c_uint64 * world)(*[b.data_ptr() for b in bufs])
    m, hd = h.shape
    return _native.lib().dqg_peer_allreduce_add_rms_norm(
        part.data_ptr(), h.data_ptr(), w.data_ptr(), y.data_ptr(), m, hd, eps, ptrs,
        ctl.data_ptr(), cap, rank, world, wait_ns, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,hd", [(1, 4096), (3, 1024), (2, 8192), (1, 8)])
def test_fused_norm_gives_the_bits_of_allreduce_then_norm(cuda_device, m, hd):
    """dqg_peer_allreduce_add_rms_norm with rank 1's packets in place: h and y
    bit-identical to the all-reduced delta followed by dqg_add_rms_norm."""
    from dequant_project_b200 import decode_ops
    cap, world = 65536, 2
    mine, peer = _buffers(cap, world, cuda_device), _buffers(cap, world, cuda_device)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(m * hd)
    a = torch.randn(m, hd, generator=g, device=cuda_device).half()
    b = torch.randn(m, hd, generator=g, device=cuda_device).half()
    h = (4 * torch.randn(m, hd, generator=g, device=cuda_device)).half()
    w = (1 + 0.1 * torch.randn(hd, generator=g, device=cuda_device)).half()
    n = m * hd
    pk = _packets(mine, cap, world)
    pk[1, 1, :n // 2, 0] = b.view(-1).view(torch.int32)
    pk[1, 1, :n // 2, 1] = 1
    h_ref = h.clone()
    y_ref = decode_ops.add_rms_norm(h_ref, (a.float() + b.float()).half(), w, 1e-5)
    y = torch.empty_like(h)
    a0 = a.clone()
    _native.device_status(cuda_device.index, reset=True)
    _native.check(_norm_call(a, h, w, y, [mine, peer], ctl, cap, 0, world))
    torch.cuda.synchronize()
    assert torch.equal(h, h_ref) and torch.equal(y, y_ref)
    assert torch.equal(a, a0)                      # the partial is left as it was
    pp = _packets(peer, cap, world)
    assert torch.equal(pp[1, 0, :n // 2, 0], a.view(-1).view(torch.int32))
    assert ctl.tolist() == [1, 0] and _native.device_status(cuda_device.index) == 0


def test_fused_norm_missing_peer_leaves_rows_alone(cuda_device):
    cap, world, m, hd = 8192, 2, 2, 4096
    mine, peer = _buffers(cap, world, cuda_device), _buffers(cap, world, cuda_device)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    a = torch.randn(m, hd, device=cuda_device).half()
    h = torch.randn(m, hd, device=cuda_device).half()
    h0 = h.clone()
    w = torch.ones(hd, dtype=torch.float16, device=cuda_device)
    y = torch.full_like(h, 3.0)
    _native.device_status(cuda_device.index, reset=True)
    _native.check(_norm_call(a, h, w, y, [mine, peer], ctl, cap, 0, world, wait_ns=20_000_000))
    torch.cuda.synchronize()
    assert _native.device_status(cuda_device.index, reset=True) & 1
    assert torch.equal(h, h0) and bool((y == 3.0).all())
    assert ctl.tolist() == [1, 0]
    bad = _norm_call(a, h, w, y, [mine, peer], ctl, 4096, 0, world)   # M * H > cap
    assert bad == 1 and b"fit cap" in _native.lib().dqg_last_error()


def test_rejects_bad_arguments(cuda_device):
    cap = 4096
    mine = _buffers(cap, 2, cuda_device)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    a = torch.zeros(cap, dtype=torch.float16, device=cuda_device)
    for kw, msg in ((dict(n=12), b"multiple of 8"), (dict(n=cap + 8), b"at most cap"),
                    (dict(rank=2), b"out of range"), (dict(wait_ns=5), b"wait_ns")):
        args = dict(n=cap, rank=0, world=2, wait_ns=0)
        args.update(kw)
        rc = _call(a, a, args["n"], [mine, mine], ctl, cap, args["rank"], args["world"],
                   args["wait_ns"])
        assert rc == 1 and msg in _native.lib().dqg_last_error()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(target, world, limit_s=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
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
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert set(out) == set(range(world)), out
    for r, (status, val) in out.items():
        assert status == "ok", val
    return {r: v for r, (_, v) in out.items()}


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_bit_exact_eager_and_graph():
    import tp_workers
    _run_ranks(tp_workers.peer_allreduce_check, 2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_decoder_peer_matches_nccl():
    import tp_workers
    out = _run_ranks(tp_workers.decoder_peer_vs_nccl, 2)
    assert torch.equal(out[0], out[1])


def _packed_layer(n, k, seed, dev):
    from dequant_project_b200.packer import QuantConfig, quantize_tensor
    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randn(n, k, generator=g, device=dev).half() * 0.02
    return quantize_tensor(w, QuantConfig(4, 128, False))


@pytest.mark.parametrize("m", (1, 8))
def test_fused_row_parallel_sums_a_ready_peer(cuda_device, m):
    """dqg_gemv_allreduce on one GPU as rank 0 of 2, the other rank's partial
    already in its exchange buffer with every CTA flag raised: y is this
    rank's fp32 partial plus the peer's, rounded once; the partial itself is
    what the plain GEMV rounds to fp16."""
    from dequant_project_b200 import dequant_cuda
    n, k, world, cap = 4096, 2048, 2, 8 * 4096
    pw = _packed_layer(n, k, 3, cuda_device)
    x = torch.randn(m, k, device=cuda_device).half()
    flags_bytes = 1024 * world * 4
    mine = torch.zeros(2 * cap * 4 + flags_bytes, dtype=torch.uint8, device=cuda_device)
    peer = torch.zeros_like(mine)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    peer_part = torch.randn(m * n, device=cuda_device)
    peer[:2 * cap * 4].view(torch.float32)[cap:cap + m * n] = peer_part   # epoch 1 -> half 1
    mine[2 * cap * 4:].view(torch.int32)[1::2] = 7                        # rank 1 is ahead
    y = torch.empty(m, n, dtype=torch.float16, device=cuda_device)
    data = (ctypes.c_uint64 * 2)(mine.data_ptr(), peer.data_ptr())
    flags = (ctypes.c_uint64 * 2)(mine.data_ptr() + 2 * cap * 4, peer.data_ptr() + 2 * cap * 4)
    _native.device_status(cuda_device.index, reset=True)
    _native.check(_native.lib().dqg_gemv_allreduce(
        x.data_ptr(), pw.qweight.data_ptr(), pw.scales.data_ptr(), pw.zeros.data_ptr(),
        y.data_ptr(), m, n, k, 4, 128, 0, 0, data, flags, ctl.data_ptr(), cap, 0, world, 0,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    part = mine[:2 * cap * 4].view(torch.float32)[cap:cap + m * n]
    assert torch.equal(y.view(-1), (part + peer_part).half())
    plain = dequant_cuda.gemv(x, pw.qweight, pw.scales, pw.zeros, 4, 128, False, False)
    assert torch.equal(part.half().view(m, n), plain)
    assert ctl.tolist() == [1, 0]
    assert _native.device_status(cuda_device.index) == 0


def test_fused_row_parallel_missing_peer_reports(cuda_device):
    n, k, world, cap = 1024, 1024, 2, 4096
    pw = _packed_layer(n, k, 4, cuda_device)
    x = torch.randn(1, k, device=cuda_device).half()
    mine = torch.zeros(2 * cap * 4 + 1024 * world * 4, dtype=torch.uint8, device=cuda_device)
    peer = torch.zeros_like(mine)
    ctl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    y = torch.full((1, n), 5.0, dtype=torch.float16, device=cuda_device)
    data = (ctypes.c_uint64 * 2)(mine.data_ptr(), peer.data_ptr())
    flags = (ctypes.c_uint64 * 2)(mine.data_ptr() + 2 * cap * 4, peer.data_ptr() + 2 * cap * 4)
    _native.device_status(cuda_device.index, reset=True)
    _native.check(_native.lib().dqg_gemv_allreduce(
        x.data_ptr(), pw.qweight.data_ptr(), pw.scales.data_ptr(), pw.zeros.data_ptr(),
        y.data_ptr(), 1, n, k, 4, 128, 0, 0, data, flags, ctl.data_ptr(), cap, 0, world,
        20_000_000, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert _native.device_status(cuda_device.index, reset=True) & 1
    assert bool((y == 5.0).all())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_fused_row_parallel():
    import tp_workers
    _run_ranks(tp_workers.fused_row_parallel_check, 2)
