"""Worker processes for the tensor-parallel tests (spawned, one per rank).

Not a test module: pytest collects only test_*.py. Each worker joins a process
group, builds its shard of a packed layer, runs the forward, and reports its
result through a queue.
"""

from __future__ import annotations

import datetime
import os
import traceback

import torch


def _cpu_linear(x, pw):
    """CPU stand-in for the GPU GEMV: x @ dequantize(pw)^T in fp32, fp16 out
    (the reference CPU path: F.linear(x, packer.dequantize(pw)))."""
    from dequant_project_b200.packer import dequantize
    w = dequantize(pw).float()
    return (x.float() @ w.t()).to(torch.float16)


def _init(rank, world, port, backend, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(rank)
        kw["device_id"] = torch.device("cuda", rank)
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist


def _layer_inputs(n, k, cfg_tuple, m, device):
    from dequant_project_b200.packer import QuantConfig, quantize_tensor
    bits, gs, sym = cfg_tuple
    g = torch.Generator().manual_seed(1234)
    w = torch.randn(n, k, generator=g, dtype=torch.float32).to(torch.float16) * 0.02
    x = torch.randn(m, k, generator=g, dtype=torch.float32).to(torch.float16)
    bias = torch.randn(n, generator=g, dtype=torch.float32).to(torch.float16) * 0.1
    pw = quantize_tensor(w.to(device), QuantConfig(bits, gs, sym))
    return pw, x.to(device), bias.to(device)


def tp_forward(rank, world, port, backend, n, k, cfg_tuple, m, queue):
    """Column-parallel (gathered) and row-parallel forward on this rank."""
    try:
        from dequant_project_b200.tensor_parallel import (ColumnParallelQuantLinear,
                                                          RowParallelQuantLinear)
        dist = _init(rank, world, port, backend, 60)
        device = torch.device("cuda", rank) if backend == "nccl" else torch.device("cpu")
        fn = None if backend == "nccl" else _cpu_linear
        pw, x, bias = _layer_inputs(n, k, cfg_tuple, m, device)
        col = ColumnParallelQuantLinear(pw, world, rank, bias=bias, gather=True, linear_fn=fn)
        y_col = col(x)
        row = RowParallelQuantLinear(pw, world, rank, bias=bias, linear_fn=fn)
        y_row = row(x[:, row.k_lo:row.k_hi].contiguous())
        queue.put((rank, "ok", y_col.cpu(), y_row.cpu()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc(), None))


def tp_rank_fails(rank, world, port, queue):
    """Rank 1 raises before the row-parallel all-reduce; rank 0 must get an
    error from its collective (peer gone / timeout), not hang."""
    try:
        from dequant_project_b200.tensor_parallel import RowParallelQuantLinear
        dist = _init(rank, world, port, "gloo", 5)
        pw, x, bias = _layer_inputs(64, 512, (4, 128, False), 1, torch.device("cpu"))
        row = RowParallelQuantLinear(pw, world, rank, bias=bias, linear_fn=_cpu_linear)
        if rank == 1:
            raise RuntimeError("injected failure on rank 1 before the all-reduce")
        row(x[:, row.k_lo:row.k_hi].contiguous())
        queue.put((rank, "completed", None, None))
    except Exception as exc:
        queue.put((rank, "error", f"{type(exc).__name__}: {exc}", None))


TINY_CFG = dict(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, intermediate=640, vocab=1000)


def decoder_step(rank, world, port, queue, fmt=(4, 64, False), cfg_kw=None, batch=2,
                 kv_len=24, tokens=(5, 977)):
    """One decode step of a small test decoder (TINY_CFG unless ``cfg_kw``)
    on this gloo rank; reports the all-gathered logits."""
    try:
        from dequant_project_b200.decoder import DecoderConfig, TPDecoder
        from dequant_project_b200.packer import QuantConfig
        dist = _init(rank, world, port, "gloo", 120)
        cfg = DecoderConfig(**(cfg_kw or TINY_CFG))
        dec = TPDecoder(cfg, QuantConfig(*fmt), world=world, rank=rank, seed=3, batch=batch,
                        kv_len=kv_len, linear_fn=_cpu_linear)
        out = dec.step(torch.tensor(list(tokens)), dec.kv_len)
        queue.put((rank, "ok", out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc()))


def decoder_step_nccl(rank, world, port, queue):
    """One decode step of the small GPU test decoder on this NCCL rank (one GPU
    per rank), eager and then replayed from a CUDA graph."""
    try:
        from dequant_project_b200.decoder import DecodeGraph, DecoderConfig, TPDecoder
        from dequant_project_b200.packer import QuantConfig
        dist = _init(rank, world, port, "nccl", 60)
        cfg = DecoderConfig(n_layers=2, hidden=1024, n_heads=8, n_kv_heads=4,
                            intermediate=2816, vocab=5000)
        dev = torch.device("cuda", rank)
        dec = TPDecoder(cfg, QuantConfig(4, 128, False), world=world, rank=rank, device=dev,
                        seed=5, batch=2, kv_len=100)
        tokens = torch.tensor([3, 4001], device=dev)
        eager = dec.step(tokens, 100).clone()
        gr = DecodeGraph(dec, 100)
        gr.tokens.copy_(tokens)
        replayed = gr.replay().clone()
        torch.cuda.synchronize(dev)
        gr.release()
        err = ((replayed.float() - eager.float()).abs().max() / eager.float().abs().max()).item()
        if err > 1e-3:
            raise AssertionError(f"graph replay differs from the eager step (rel {err})")
        queue.put((rank, "ok", eager.cpu()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc()))


def decoder_rank_fails(rank, world, port, queue):
    """Rank 1 raises before its first decode step; rank 0's step must end with
    an error from its first collective (peer gone or timeout), not hang."""
    try:
        from dequant_project_b200.decoder import DecoderConfig, TPDecoder
        from dequant_project_b200.packer import QuantConfig
        _init(rank, world, port, "gloo", 5)
        cfg = DecoderConfig(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, intermediate=640,
                            vocab=1000)
        dec = TPDecoder(cfg, QuantConfig(4, 64, False), world=world, rank=rank, seed=3,
                        batch=1, kv_len=8, linear_fn=_cpu_linear)
        if rank == 1:
            raise RuntimeError("injected failure on rank 1 before the decode step")
        dec.step(torch.tensor([5]), 8)
        queue.put((rank, "completed", None))
    except Exception as exc:
        queue.put((rank, "error", f"{type(exc).__name__}: {exc}"))


def peer_allreduce_check(rank, world, port, queue):
    """The peer all-reduce on this NCCL rank: several sizes eagerly, then the
    same calls replayed twice from a CUDA graph; each result must equal the
    fp32 sum of every rank's input in rank order, rounded once (bit-exact)."""
    try:
        from dequant_project_b200.peer_reduce import PeerAllReduce
        dist = _init(rank, world, port, "nccl", 60)
        dev = torch.device("cuda", rank)
        ar = PeerAllReduce(None, dev, 65536)

        def inputs(seed, n):
            g = torch.Generator(device=dev).manual_seed(seed)
            return [torch.randn(n, generator=g, device=dev).half() for _ in range(world)]

        def expect(xs):
            acc = torch.zeros_like(xs[0], dtype=torch.float32)
            for x in xs:
                acc += x.float()
            return acc.half()

        sizes = [8, 4096, 8192, 2 * 2048 + 24, 65536]
        for i, n in enumerate(sizes):
            xs = inputs(100 + i, n)
            t = xs[rank].clone()
            ar(t)
            torch.cuda.synchronize(dev)
            if not torch.equal(t, expect(xs)):
                raise AssertionError(f"eager n={n}: not the rank-ordered fp32 sum")
        bufs = [inputs(200 + i, n)[rank].clone() for i, n in enumerate(sizes)]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        work = [b.clone() for b in bufs]
        with torch.cuda.graph(g, stream=side):
            for w in work:
                ar(w)
        for rep in range(2):
            for w, b in zip(work, bufs):
                w.copy_(b)
            g.replay()
            torch.cuda.synchronize(dev)
            for i, (w, n) in enumerate(zip(work, sizes)):
                if not torch.equal(w, expect(inputs(200 + i, n))):
                    raise AssertionError(f"graph replay {rep} n={n}: wrong sum")
        g.reset()
        from dequant_project_b200 import _native
        if _native.device_status(rank) != 0:
            raise AssertionError("a wait gave up")
        ar.close()
        queue.put((rank, "ok", None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc()))


def decoder_peer_vs_nccl(rank, world, port, queue):
    """The small GPU test decoder on this NCCL rank with the peer all-reduce
    (inside the following norm, and as its own kernel: the same bits) and with
    NCCL's; within 5e-3 of each other (the peer sum rounds once, NCCL's fp16
    sum per step). Reports the peer decoder's logits."""
    try:
        from dequant_project_b200.decoder import DecodeGraph, DecoderConfig, TPDecoder
        from dequant_project_b200.packer import QuantConfig
        dist = _init(rank, world, port, "nccl", 60)
        cfg = DecoderConfig(n_layers=2, hidden=1024, n_heads=8, n_kv_heads=4,
                            intermediate=2816, vocab=5000)
        dev = torch.device("cuda", rank)
        tokens = torch.tensor([3, 4001], device=dev)
        outs = {}
        for mode in ("peer", "peer_unfused", "fused", "nccl"):
            dec = TPDecoder(cfg, QuantConfig(4, 128, False), world=world, rank=rank, device=dev,
                            seed=5, batch=2, kv_len=100, allreduce=mode.split("_")[0],
                            fuse_norm=mode != "peer_unfused")
            eager = dec.step(tokens, 100).clone()
            gr = DecodeGraph(dec, 100)
            gr.tokens.copy_(tokens)
            rep = gr.replay().clone()
            torch.cuda.synchronize(dev)
            gr.release()
            dec.close()
            if not torch.equal(rep, eager):
                raise AssertionError(f"{mode}: graph replay differs from the eager step")
            outs[mode] = eager
        # The all-reduce inside the norm kernel gives the bits of the two calls.
        if not torch.equal(outs["peer"], outs["peer_unfused"]):
            raise AssertionError("fused all-reduce + norm differs from the separate calls")
        b = outs["nccl"].float()
        for mode in ("peer", "fused"):
            a = outs[mode].float()
            err = ((a - b).abs().max() / b.abs().max()).item()
            if err > 5e-3:
                raise AssertionError(f"{mode} vs nccl decoder logits differ by {err}")
        queue.put((rank, "ok", outs["peer"].cpu()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc()))


class FakeIpc:
    """Stand-in for CUDA IPC on CPU ranks: a handle names (rank, pointer);
    opening returns a fake base and records what was opened and closed."""

    def __init__(self, rank):
        self.rank, self.opened, self.closed = rank, [], []

    def export(self, ptr):
        return f"rank{self.rank}:{ptr}".encode().ljust(64, b"\0"), 16

    def open(self, handle):
        self.opened.append(handle.rstrip(b"\0").decode())
        return 1 << 40 | len(self.opened) << 20

    def close(self, base):
        self.closed.append(base)


def peer_exchange(rank, world, port, queue):
    """PeerAllReduce's set-up on gloo CPU ranks with FakeIpc: reports which
    handles this rank opened and the pointer tables it built."""
    try:
        from dequant_project_b200.peer_reduce import PeerAllReduce
        dist = _init(rank, world, port, "gloo", 60)
        ipc = FakeIpc(rank)
        ar = PeerAllReduce(None, torch.device("cpu"), 5000, ipc=ipc)
        info = {"opened": list(ipc.opened), "bufs": list(ar.peer_bufs),
                "data": list(ar.peer_data), "gemv_flags": list(ar.peer_gemv_flags),
                "own": ar.buffer.data_ptr(), "cap": ar.cap, "nbytes": ar.buffer.numel()}
        ar.close()
        ar.close()
        info["closed"] = len(ipc.closed)
        try:
            ar(torch.zeros(8, dtype=torch.float16))
            info["after_close"] = "accepted"
        except RuntimeError as exc:
            info["after_close"] = str(exc)
        queue.put((rank, "ok", info))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc()))


def fused_row_parallel_check(rank, world, port, queue):
    """PeerAllReduce.gemv on this NCCL rank (INT4 g128 row-parallel layers,
    M = 1 and 8, several calls and a graph replay): every rank gets the same
    bits, within 2e-3 of the fp32 product over the full input dimension."""
    try:
        from dequant_project_b200.packer import QuantConfig, dequantize, quantize_tensor
        from dequant_project_b200.peer_reduce import PeerAllReduce
        from dequant_project_b200.tensor_parallel import shard_rows
        dist = _init(rank, world, port, "nccl", 60)
        dev = torch.device("cuda", rank)
        ar = PeerAllReduce(None, dev, 8 * 4096)
        for i, (n, k, m) in enumerate(((4096, 4096, 1), (4096, 11008, 8), (4096, 4096, 8))):
            g = torch.Generator(device=dev).manual_seed(50 + i)
            w = torch.randn(n, k, generator=g, device=dev).half() * 0.02
            x = torch.randn(m, k, generator=g, device=dev).half()
            pw = quantize_tensor(w, QuantConfig(4, 128, False))
            shard, lo, hi = shard_rows(pw, world, rank)
            y = ar.gemv(x[:, lo:hi].contiguous(), shard)
            torch.cuda.synchronize(dev)
            ref = x.float() @ dequantize(pw).float().t()
            err = ((y.float() - ref).abs().max() / ref.abs().max()).item()
            if err > 2e-3:
                raise AssertionError(f"case {i}: rel err {err}")
            ys = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(ys, y)
            if any(not torch.equal(ys[0], t) for t in ys):
                raise AssertionError(f"case {i}: ranks disagree")
        from dequant_project_b200 import _native
        if _native.device_status(rank) != 0:
            raise AssertionError("a wait gave up")
        ar.close()
        queue.put((rank, "ok", None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "error", traceback.format_exc()))
