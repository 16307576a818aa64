"""Decode ms/token of the tensor-parallel packed decoder.

    python -m dequant_project_b200.decode_bench [--model llama2-7b] [--bits 4]
        [--group-size 128] [--batch 1] [--kv-len 2048] [--steps 50] [--warmup 5]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m dequant_project_b200.decode_bench ...
    python -m dequant_project_b200.decode_bench --model llama3-70b --save-weights m.pt
    python -m dequant_project_b200.decode_bench --weights m.pt     # no quantization

One process per GPU; the tensor-parallel width is the world size. The model
(random N(0, 0.02) weights, every linear packed, N(0, 1) fp16 KV cache of
``kv_len`` positions) is built on each rank, one decode step at position
``kv_len`` is captured in a CUDA graph, and ``steps`` replays are timed with
CUDA events on the replay stream after ``warmup`` untimed ones, bracketed by a
barrier; the time is the maximum over ranks. Each replay rewrites the same
cache slot, so every timed step does identical work. Rank 0 prints one JSON
line: ms/token, tokens/s, and the step's bytes on one rank (packed weights, KV
cache, embedding row, norms) over the time against the measured HBM copy
bandwidth.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch

MODELS = {"llama2-7b": "LLAMA2_7B", "llama3-70b": "LLAMA3_70B"}


def measure(args, dist, rank: int, world: int, dev: torch.device) -> dict | None:
    """Build this rank's shard, capture and time the step (see the module
    text) inside an existing process group (``dist`` is None for one GPU).
    Every rank takes the same collective steps; rank 0 returns the result
    line, the others None."""
    from dequant_project_b200 import decoder as D
    from dequant_project_b200.byte_model import measured_peaks

    local = dev.index
    cfg, q, weights = model_source(args, dev)
    dec = D.TPDecoder(cfg, q, world=world, rank=rank, device=dev, seed=args.seed,
                      batch=args.batch, kv_len=args.kv_len, weights=weights)
    del weights
    torch.cuda.synchronize(dev)
    gr = D.DecodeGraph(dec, args.kv_len)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        gr.replay()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier(device_ids=[local])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("decode_timed")   # lets a profiler select the timed replays
    e0.record(stream)
    for _ in range(args.steps):
        gr.replay()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier(device_ids=[local])
    by = dec.step_bytes(args.kv_len)
    gr.release()
    del gr, dec
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peaks = measured_peaks()
    gbs = by["total"] / (ms * 1e-3) / 1e9
    return {
        "metric": "decode ms/token", "value": round(ms, 4), "unit": "ms/token",
        "tokens_per_s": round(args.batch / (ms * 1e-3), 1), "n_gpus": world,
        "tp": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": False,
        "config": {"model": args.model if not getattr(args, "weights", None) else args.weights,
                   "layers": cfg.n_layers, "batch": args.batch,
                   "kv_len": args.kv_len, "bits": q.bits,
                   "group_size": q.group_size or "per-channel",
                   "symmetric": q.symmetric, "lm_head": "packed, column-parallel"},
        "data": "synthetic (random-init N(0,0.02) weights, N(0,1) fp16 KV cache)",
        "bytes_per_rank": by,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "floor_ms": round(by["total"] / (peaks["hbm_gbs"] * 1e9) * 1e3, 4)},
    }


def model_source(args, device):
    """(DecoderConfig, QuantConfig, weights): the packed file ``args.weights``
    when given (its configuration wins), else the named model drawn from
    ``args.seed``."""
    from dequant_project_b200 import decoder as D
    from dequant_project_b200.packer import QuantConfig

    if getattr(args, "weights", None):
        model = D.PackedModel.load(args.weights, device=device)
        return model.cfg, model.qcfg, model
    cfg = getattr(D, MODELS[args.model])
    if args.layers:
        cfg = D.DecoderConfig(args.layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads,
                              cfg.intermediate, cfg.vocab, cfg.rope_theta, cfg.eps)
    return cfg, QuantConfig(args.bits, args.group_size or None, args.sym), None


def save_model(args, device) -> None:
    """Pack the named model once (on ``device``) and write it to
    ``args.save_weights``, for later runs with ``--weights``."""
    from dequant_project_b200 import decoder as D

    cfg, q, _ = model_source(argparse.Namespace(**{**vars(args), "weights": None}), device)
    D.PackedModel.build(cfg, q, seed=args.seed, device=device).save(args.save_weights)


def run(args) -> dict | None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    try:
        return measure(args, dist, rank, world, dev)
    finally:
        if dist is not None:
            dist.destroy_process_group()


def default_args(**kw) -> argparse.Namespace:
    """The CLI's defaults (Llama-2-7B, INT4 g128 asym, batch 1, 2048-token
    cache), overridden by ``kw``."""
    ns = _parser().parse_args([])
    for k, v in kw.items():
        setattr(ns, k, v)
    return ns


def _parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", choices=sorted(MODELS), default="llama2-7b")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count")
    ap.add_argument("--bits", type=int, default=4, choices=(2, 4, 8))
    ap.add_argument("--group-size", type=int, default=128, help="0 = per-channel")
    ap.add_argument("--sym", action="store_true")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--kv-len", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--weights", default=None,
                    help="load the packed model from this file (packed_io format)")
    ap.add_argument("--save-weights", default=None,
                    help="pack the model once, write it to this file and exit")
    return ap


def main() -> None:
    args = _parser().parse_args()
    if args.save_weights:
        save_model(args, torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
        return
    line = run(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
