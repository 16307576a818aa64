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


def decoder_step(rank, world, port, queue, fmt=(4, 64, False)):
    """One decode step of the tiny test decoder on this gloo rank."""
    try:
        from dequant_project_b200.decoder import DecoderConfig, TPDecoder
        from dequant_project_b200.packer import QuantConfig
        dist = _init(rank, world, port, "gloo", 60)
        cfg = DecoderConfig(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, intermediate=640,
                            vocab=1000)
        dec = TPDecoder(cfg, QuantConfig(*fmt), world=world, rank=rank, seed=3, batch=2,
                        kv_len=24, linear_fn=_cpu_linear)
        out = dec.step(torch.tensor([5, 977]), dec.kv_len)
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
