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


def _time_graph(graph_fn, steps: int, warmup: int, dev, dist=None) -> float:
    """ms per replay of a CUDA graph (``graph_fn`` replays once), CUDA events
    on the current stream after ``warmup`` replays, max over ranks."""
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, warmup)):
        graph_fn()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier(device_ids=[dev.index])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph_fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _capture(fn, dev):
    """A CUDA graph of ``fn()`` (side-stream warm-up first)."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def gemv_only(dec, dev) -> tuple:
    """(graph, launches, bytes) of the step's packed GEMVs alone, with the
    step's shapes and weights in the step's order (static random inputs)."""
    from dequant_project_b200 import quant_linear as ql
    from dequant_project_b200.byte_model import gemv_bytes
    from dequant_project_b200.packer import PackedWeight

    m = dec.batch
    mats = [w[k] for w in dec.layers for k in ("qkv", "o", "gu", "down")]
    if isinstance(dec.lm_head, PackedWeight):
        mats.append(dec.lm_head)
    xs = [torch.randn(m, pw.shape[1], device=dev, dtype=torch.float16) for pw in mats]
    nbytes = sum(gemv_bytes(pw.shape[0], pw.shape[1], pw.config.bits, pw.config.group_size,
                            pw.config.symmetric, m) for pw in mats)

    def run():
        for x, pw in zip(xs, mats):
            ql.gemv(x, pw)

    return _capture(run, dev), len(mats), nbytes


def attention_only(dec, dev, pos: int) -> tuple:
    """(graph, bytes) of the step's attention calls alone (every layer's
    cache, positions 0..pos)."""
    from dequant_project_b200 import decode_ops as ops

    d = dec.cfg.head_dim
    q = torch.randn(dec.batch, dec.hq, d, device=dev, dtype=torch.float16)

    def run():
        for kc, vc in zip(dec.k_cache, dec.v_cache):
            ops.attention(q, kc, vc, pos + 1, dec._attn_ws)

    nbytes = dec.cfg.n_layers * 2 * dec.batch * dec.hkv * (pos + 1) * d * 2
    return _capture(run, dev), nbytes


def allreduce_only(dec, dev) -> tuple:
    """(graph, launches) of the step's all-reduces alone: two per layer over
    [batch, hidden] fp16, through the decoder's collective (world > 1)."""
    t = torch.randn(dec.batch, dec.cfg.hidden, device=dev, dtype=torch.float16)
    n = 2 * dec.cfg.n_layers

    def run():
        for _ in range(n):
            dec._all_reduce(t)

    return _capture(run, dev), n


def measure(args, dist, rank: int, world: int, dev: torch.device, parts: bool = True,
            e2e: bool = True, check_tp1: bool = False) -> dict | None:
    """Build this rank's shard, capture and time the step (see the module
    text) inside an existing process group (``dist`` is None for one GPU).
    With ``parts``, the step's GEMVs alone and its attention alone are timed
    too (their own graphs, same shapes and weights); with ``e2e``, the step is
    also timed end to end as a caller runs it (token ids copied in from pinned
    host memory, the step's graph replayed, the logits copied back to pinned
    host memory, every step); with ``check_tp1`` (world > 1), rank 0 rebuilds
    the model on one GPU and compares the logits. Every rank takes the same
    collective steps; rank 0 returns the result line, the others None."""
    from dequant_project_b200 import decoder as D
    from dequant_project_b200.byte_model import measured_peaks

    cfg, q, weights = model_source(args, dev)
    dec = D.TPDecoder(cfg, q, world=world, rank=rank, device=dev, seed=args.seed,
                      batch=args.batch, kv_len=args.kv_len, weights=weights,
                      allreduce=getattr(args, "allreduce", "peer"),
                      l2_prefetch=getattr(args, "l2_prefetch", False))
    torch.cuda.synchronize(dev)
    gr = D.DecodeGraph(dec, args.kv_len)
    gr.tokens.copy_(torch.arange(args.batch, device=dev) * 7919 % cfg.vocab)
    torch.cuda.nvtx.range_push("decode_timed")   # lets a profiler select the timed replays
    ms = _time_graph(gr.replay, args.steps, args.warmup, dev, dist)
    torch.cuda.nvtx.range_pop()
    logits = gr.replay().float()
    torch.cuda.synchronize(dev)
    out_e2e = None
    if e2e:
        tok_host = torch.zeros(args.batch, dtype=torch.int64).pin_memory()
        tok_host.copy_(gr.tokens.cpu())
        logit_host = torch.empty(tuple(logits.shape), dtype=torch.float16).pin_memory()

        def e2e_step():
            gr.tokens.copy_(tok_host, non_blocking=True)
            gr.replay()
            logit_host.copy_(gr.logits, non_blocking=True)

        ms_e2e = _time_graph(e2e_step, max(1, args.steps // 2), args.warmup, dev, dist)
        out_e2e = {"ms_per_token": round(ms_e2e, 4),
                   "tokens_per_s": round(args.batch / (ms_e2e * 1e-3), 2),
                   "h2d_bytes_per_step": tok_host.numel() * 8,
                   "d2h_bytes_per_step": logit_host.numel() * 2}
    gemv_part = attn_part = ar_part = None
    if parts:
        g_gemv, launches, gbytes = gemv_only(dec, dev)
        ms_g = _time_graph(g_gemv.replay, args.steps, args.warmup, dev, dist)
        g_gemv.reset()
        gemv_part = {"ms": ms_g, "launches": launches, "bytes": gbytes}
        if dev.type == "cuda" and cfg.head_dim == 128:
            g_att, abytes = attention_only(dec, dev, args.kv_len)
            ms_a = _time_graph(g_att.replay, args.steps, args.warmup, dev, dist)
            g_att.reset()
            attn_part = {"ms": ms_a, "launches": cfg.n_layers, "bytes": abytes}
        if world > 1:
            g_ar, n_ar = allreduce_only(dec, dev)
            ms_r = _time_graph(g_ar.replay, args.steps, args.warmup, dev, dist)
            g_ar.reset()
            ar_part = {"ms": ms_r, "launches": n_ar,
                       "bytes": n_ar * args.batch * cfg.hidden * 2}
    by = dec.step_bytes(args.kv_len)
    gr.release()
    dec.close()
    del gr, dec
    torch.cuda.empty_cache()
    tp1_err = None
    if check_tp1 and world > 1 and rank == 0:
        one = D.TPDecoder(cfg, q, world=1, rank=0, device=dev, seed=args.seed, batch=args.batch,
                          kv_len=args.kv_len, weights=weights)
        toks = torch.arange(args.batch, device=dev) * 7919 % cfg.vocab
        ref = one.step(toks, args.kv_len).float()
        tp1_err = ((logits - ref).abs().max() / ref.abs().max()).item()
        del one, ref
        torch.cuda.empty_cache()
    del weights
    if dist is not None:
        dist.barrier(device_ids=[dev.index])
    if rank != 0:
        return None
    peaks = measured_peaks()
    gbs = by["total"] / (ms * 1e-3) / 1e9
    line = {
        "metric": "decode ms/token", "value": round(ms, 4), "unit": "ms/token",
        "tokens_per_s": round(args.batch / (ms * 1e-3), 1), "n_gpus": world,
        "tp": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": False,
        "config": {"model": args.weights if getattr(args, "weights", None) else args.model,
                   "layers": cfg.n_layers, "batch": args.batch,
                   "kv_len": args.kv_len, "bits": q.bits,
                   "group_size": q.group_size or "per-channel",
                   "symmetric": q.symmetric, "lm_head": "packed, column-parallel",
                   "allreduce": getattr(args, "allreduce", "peer") if world > 1 else None,
                   "l2_prefetch": getattr(args, "l2_prefetch", False)},
        "data": "synthetic (random-init N(0,0.02) weights, N(0,1) fp16 KV cache)",
        "bytes_per_rank": by,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "floor_ms": round(by["total"] / (peaks["hbm_gbs"] * 1e9) * 1e3, 4)},
        "logits_checksum": round(float(logits.double().sum()), 3),
    }
    if out_e2e is not None:
        line["e2e"] = out_e2e
    for name, part in (("gemv", gemv_part), ("attention", attn_part)):
        if part is not None:
            a = part["bytes"] / (part["ms"] * 1e-3) / 1e9
            line[name] = {"ms_per_step": round(part["ms"], 4), "launches": part["launches"],
                          "us_per_launch": round(part["ms"] * 1e3 / part["launches"], 3),
                          "bytes_per_step": part["bytes"], "achieved_gbs": round(a, 1),
                          "frac": round(a / peaks["hbm_gbs"], 4),
                          "share_of_step": round(part["ms"] / ms, 3)}
    if ar_part is not None:
        line["allreduce"] = {"ms_per_step": round(ar_part["ms"], 4),
                             "launches": ar_part["launches"],
                             "us_per_launch": round(ar_part["ms"] * 1e3 / ar_part["launches"], 3),
                             "bytes_per_launch": ar_part["bytes"] // ar_part["launches"],
                             "share_of_step": round(ar_part["ms"] / ms, 3)}
    if tp1_err is not None:
        # 32 random layers amplify the fp16 rounding differences of another
        # summation order (partial sums per rank); the gloo tests bound the
        # kernels' own arithmetic at 5e-3 on two layers.
        line["tp1_check"] = {"max_rel_err_vs_tp1": tp1_err, "tolerance": 2e-2,
                             "ok": tp1_err <= 2e-2}
    return line


def model_source(args, device):
    """(DecoderConfig, QuantConfig, weights): the packed file ``args.weights``
    when given (its configuration wins), else the named model drawn from
    ``args.seed``."""
    from dequant_project_b200 import decoder as D
    from dequant_project_b200.packer import QuantConfig

    if getattr(args, "packed_model", None) is not None:
        model = args.packed_model
        return model.cfg, model.qcfg, model
    if getattr(args, "weights", None):
        # Host memory, memory-mapped: each rank moves only its shards to its
        # GPU (TPDecoder shards one full matrix at a time).
        model = D.PackedModel.load(args.weights, device=None)
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
    from dequant_project_b200 import _native
    _native.lib().dqg_set_gemv_path(args.gemv_path)
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
        return measure(args, dist, rank, world, dev, check_tp1=args.check_tp1)
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
    ap.add_argument("--l2-prefetch", action="store_true",
                    help="L2 prefetch of later GEMVs' weights in the element-wise ops")
    ap.add_argument("--allreduce", choices=("peer", "fused", "nccl"), default="peer",
                    help="collective after the row-parallel layers (world > 1)")
    ap.add_argument("--gemv-path", type=int, default=0, choices=(0, 1),
                    help="dqg_set_gemv_path: 0 = per shape (default), 1 = no direct kernel")
    ap.add_argument("--check-tp1", action="store_true",
                    help="rank 0 compares the logits with the model on one GPU")
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
