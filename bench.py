#!/usr/bin/env python
"""Benchmark of the fused low-bit dequant + GEMV decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU)

Headline (every N): decode tokens/s of a Llama-2-7B
architecture decoder whose every linear layer and the LM head are INT4 g128
packed, batch 1, 2048-token fp16 KV cache, tensor-parallel over the N ranks
(column-parallel QKV and gate/up, row-parallel O and down with an all-reduce
over peer memory, vocabulary-parallel LM head). One step = one token; the
same model and token at every N, so ``scaling`` is "strong" and the driver's
efficiency is the decode step's. Weights are random-init ~N(0, 0.02) (no
checkpoints offline), 3.5 GB packed: far larger than the 126 MB L2. The step
is replayed from a CUDA graph, timed with CUDA events, max over ranks.

``roofline`` is the dominant kernel of that step, the fused dequant + GEMV:
the step's GEMVs alone (same shapes, weights and order, their own graph),
algorithmic bytes over device time against the measured HBM copy bandwidth.
``e2e`` is the same step as a caller runs it: token ids copied in from pinned
host memory, the graph replayed, the logits copied back to pinned host memory.

Sub-keys: ``decode_batch8`` (same model, batch 8); ``decode_70b`` (N >= 2,
Llama-3-70B architecture, INT4 g128 and INT2 g64, batch 1
and 8, 4096-token cache); ``gemv_sweep`` (N = 1: the 18
bit-width sweep GEMVs as one graph, with per-case µs, and ``shape_sweep``,
BASELINE config 3; both also time the reference's own CUDA kernel, built
unmodified for sm_100a by baseline/build_reference_kernel.py, on the same
cases).

``--impl reference`` times the reference's CPU path for the same token (its
GEMVs ``F.linear(x, packer.dequantize(W))`` as the C restatement in oracle/,
all host threads) on a bounded row sample of every matrix of one layer and the
LM head, scaled to the whole step; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("decode tokens/s, Llama-2-7B architecture, all linears and LM head INT4 g128 "
          "packed, batch 1, 2048-token KV cache, tensor-parallel over n_gpus")
UNIT = "tokens/s"
SWEEP_METRIC = ("GEMV achieved HBM GB/s over the bit-width sweep "
                "(INT8 per-ch / INT4 g128 / INT2 g64; 4096x11008 & 11008x4096; M=1,4,8)")
SHAPES = [(4096, 11008), (11008, 4096)]
FORMATS = [(8, None, True, "int8-perch-sym"), (4, 128, False, "int4-g128-asym"),
           (2, 64, False, "int2-g64-asym")]
BATCHES = (1, 4, 8)


def cases():
    return [(n, k, bits, gs, sym, m, name)
            for (n, k) in SHAPES for (bits, gs, sym, name) in FORMATS for m in BATCHES]


def case_bytes(n, k, bits, gs, sym, m):
    from dequant_project_b200.byte_model import gemv_bytes
    return gemv_bytes(n, k, bits, gs, sym, m)


def workload_config(world):
    return {"workload": "decode step (BASELINE config 4): Llama-2-7B architecture, INT4 g128 "
                        "(asymmetric) linears and LM head, batch 1, 2048-token fp16 KV cache",
            "tokens_per_step": 1,
            "l2": "inputs > L2 (3.5 GB of packed weights and 1.07 GB of KV cache per step)",
            "parallelism": f"tp{world}" if world > 1 else "tp1"}


def sweep_config():
    return {"workload": "bit-width sweep (BASELINE config 2): 18 GEMVs/step",
            "shapes": ["4096x11008", "11008x4096"],
            "formats": [f[3] for f in FORMATS], "batches": list(BATCHES),
            "l2": "inputs > L2 (18 distinct packed matrices, ~480 MB per step)"}


# --------------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a thread."""

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.dev = device_index
        self.period = period_s
        self.samples = []   # (t, sm_mhz, reasons_bitmask)
        self._stop = threading.Event()
        self._thr = None
        self.max_mhz = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are diagnostics, never fatal
            return self
        self._thr = threading.Thread(target=self._run, daemon=True)
        self._thr.start()
        return self

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr:
            self._thr.join()
        return False

    def summary(self, t0: float, t1: float):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        used = inside if len(inside) >= 3 else self.samples
        names = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}
        mask = 0
        for s in used:
            mask |= s[2]
        return {"sm_mhz": statistics.median(s[1] for s in used) if used else None,
                "sm_max_mhz": self.max_mhz,
                "reasons": [v for b, v in names.items() if mask & b and b != 0x1],
                "samples": len(used), "samples_in_timed_region": len(inside)}


# ------------------------------------------------------------------ our arm

def gemv_sweep(args, dev, peaks):
    """BASELINE config 2 on this GPU: the 18 sweep GEMVs, each on its own
    packed tensors, replayed from one graph; GB/s over device time, per-case
    µs, the shape sweep, and the same through the public call with host
    buffers."""
    import torch

    from dequant_project_b200 import dequant_cuda
    from dequant_project_b200.packer import QuantConfig, quantize_tensor

    cs = cases()
    data = []
    for i, (n, k, bits, gs, sym, m, _) in enumerate(cs):
        g = torch.Generator(device=dev).manual_seed(1000 + i)
        w = torch.randn(n, k, dtype=torch.float16, device=dev, generator=g) * 0.02
        pw = quantize_tensor(w, QuantConfig(bits, gs, sym))
        del w
        x = torch.randn(m, k, dtype=torch.float16, device=dev, generator=g)
        data.append((pw, x))
    torch.cuda.synchronize()
    step_bytes = sum(case_bytes(n, k, bits, gs, sym, m) for (n, k, bits, gs, sym, m, _) in cs)

    def step():
        for (n, k, bits, gs, sym, m, _), (pw, x) in zip(cs, data):
            dequant_cuda.gemv(x, pw.qweight, pw.scales, pw.zeros, bits, gs or k, sym, False)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    del graph
    gbs = step_bytes / (ms * 1e-3) / 1e9
    out = {"metric": SWEEP_METRIC, "value": round(gbs, 2), "unit": "GB/s",
           "ms_per_step": round(ms, 5), "config": sweep_config(),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                        "bytes_per_launch_avg": step_bytes // len(cs)}}
    e2e = run_e2e(dev, cs, data, args, None, dev.index)
    out["e2e"] = {"value": round(step_bytes / (e2e["ms"] * 1e-3) / 1e9, 2), "unit": "GB/s",
                  "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                  "path": "dequant_cuda.gemv (eager, pinned host x -> device -> pinned host y)"}
    if not args.no_detail:
        out["detail"] = per_case_detail(dev, cs, data, peaks)
        try:
            out["reference_kernel"] = reference_kernel_detail(dev, cs, data, peaks, out["detail"])
        except Exception as exc:  # noqa: BLE001 - reported, never fatal to the line
            out["reference_kernel"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        try:
            out["shape_sweep"] = shape_sweep(dev, peaks, with_reference=True)
        except Exception as exc:  # noqa: BLE001 - reported, never fatal to the line
            out["shape_sweep"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    if not args.no_cpu:
        out["cpu_baseline"] = cpu_baseline(cs, data, budget_s=args.cpu_seconds / 2)
    del data
    torch.cuda.empty_cache()
    return out


def decode_launches(cfg, world: int) -> int:
    """Launches of this library's kernels in one decode step of the default
    decoder: per layer two norms (at world > 1 each with the all-reduce of the
    row-parallel output before it inside), the QKV, O and down GEMVs, the
    gate/up GEMV with its SwiGLU, RoPE + KV append and attention; then the
    final norm and the LM head GEMV. ``world`` does not change the count."""
    del world
    return cfg.n_layers * 8 + 2


def run_ours(args, rank, world, local_rank):
    import torch

    from dequant_project_b200 import decode_bench
    from dequant_project_b200 import decoder as D
    from dequant_project_b200.byte_model import measured_peaks

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    peaks = measured_peaks()

    # Headline: BASELINE config 4 at TP = world, clocks sampled throughout.
    dargs = decode_bench.default_args(steps=args.steps, warmup=args.warmup)
    with ClockSampler(local_rank) as clk:
        t0 = time.perf_counter()
        line = decode_bench.measure(dargs, dist, rank, world, dev, parts=True, e2e=True,
                                    check_tp1=world > 1)
        t1 = time.perf_counter()
    extra = {}
    if not args.no_decode:
        try:
            extra["decode_batch8"] = decode_bench.measure(
                decode_bench.default_args(steps=max(20, args.steps // 4), warmup=args.warmup,
                                          batch=8), dist, rank, world, dev, parts=False,
                e2e=False)
        except Exception as exc:  # noqa: BLE001 - reported, never fatal to the line
            extra["decode_batch8"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        if world > 1 or args.with_70b:
            extra["decode_70b"] = decode_70b(args, dist, rank, world, dev)
    sweep = None
    if world == 1 and not args.no_sweep:
        sweep = gemv_sweep(args, dev, peaks)
    if rank == 0:
        ms = line["value"]
        tps = 1.0 / (ms * 1e-3)
        gemv = line.get("gemv", {})
        out = {
            "metric": METRIC, "value": round(tps, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 activations x int4 codes, fp32 accumulate",
            "data": "synthetic (random-init N(0,0.02) weights, N(0,1) fp16 KV cache)",
            "config": workload_config(world),
            "roofline": {"bound": "hbm", "kernel": "the step's fused dequant + GEMV launches "
                                                  "(dqg direct kernel), timed alone",
                         "achieved": gemv.get("achieved_gbs"), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": gemv.get("frac"),
                         "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, copy)",
                         "bytes_per_launch_avg": (gemv["bytes_per_step"] // gemv["launches"]
                                                  if gemv else None),
                         "us_per_launch": gemv.get("us_per_launch"),
                         "traffic": load_traffic()},
            "e2e": {"value": line["e2e"]["tokens_per_s"], "unit": UNIT,
                    "h2d_bytes_per_step": line["e2e"]["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": line["e2e"]["d2h_bytes_per_step"],
                    "ms_per_step": line["e2e"]["ms_per_token"],
                    "path": "DecodeGraph: token ids from pinned host, graph replay, logits to "
                            "pinned host, every step"},
            "gpu_launches": decode_launches(D.LLAMA2_7B, world) * args.steps,
            "clocks": clk.summary(t0, t1),
            "cpu_baseline": (cpu_decode_baseline(args.cpu_seconds)
                             if world == 1 and not args.no_cpu else None),
            "decode": line,
            **extra,
            "gemv_sweep": sweep,
        }
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def decode_70b(args, dist, rank, world, dev):
    """BASELINE config 5 at TP = world: Llama-3-70B architecture, INT4 g128
    and INT2 g64, batch 1 and 8, 4096-token cache. Each format is packed once
    per rank (PackedModel) and shared by the two batch sizes."""
    import torch

    from dequant_project_b200 import decode_bench
    from dequant_project_b200 import decoder as D
    from dequant_project_b200.packer import QuantConfig

    out = {}
    for bits, gs in ((4, 128), (2, 64)):
        key = f"int{bits}_g{gs}"
        try:
            model = D.PackedModel.build(D.LLAMA3_70B, QuantConfig(bits, gs, False), seed=0,
                                        device=dev)
            for batch in (1, 8):
                a = decode_bench.default_args(model="llama3-70b", bits=bits, group_size=gs,
                                              batch=batch, kv_len=4096,
                                              steps=max(10, args.steps // 10),
                                              warmup=args.warmup)
                a.packed_model = model
                r = decode_bench.measure(a, dist, rank, world, dev, parts=False, e2e=False)
                if r is not None:
                    out[f"{key}_b{batch}"] = {k: r[k] for k in ("value", "unit", "tokens_per_s",
                                                                "roofline", "bytes_per_rank")}
            del model
        except Exception as exc:  # noqa: BLE001 - reported, never fatal to the line
            out[key] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        torch.cuda.empty_cache()
    return out if rank == 0 else None


SHAPE_SWEEP = [(4096, 4096), (12288, 4096), (4096, 14336), (28672, 8192), (8192, 28672),
               (128256, 4096)]


REF_KERNEL = ROOT / "baseline" / "_ref" / "ext" / "dequant_cuda_ref.so"


def reference_kernel():
    """The reference's own CUDA extension built for sm_100a by
    baseline/build_reference_kernel.py, or None when it is not built."""
    if not REF_KERNEL.exists():
        return None
    import importlib.util
    spec = importlib.util.spec_from_file_location("dequant_cuda_ref", REF_KERNEL)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_kernel_detail(dev, cs, data, peaks, ours):
    """µs per case of the reference kernel (kernels/dequant_gemv.cu:144-217,
    unmodified, compiled for sm_100a) measured exactly like ``detail``, with
    this library's µs beside it."""
    mod = reference_kernel()
    if mod is None:
        return {"error": "reference kernel not built (python baseline/build_reference_kernel.py "
                         "REFERENCE_ROOT)"}
    rows = per_case_detail(dev, cs, data, peaks, reps=10, gemv_fn=mod.gemv)
    ours_us = {r["case"]: r["us"] for r in ours}
    for r in rows:
        r["ours_us"] = ours_us.get(r["case"])
        r["speedup"] = round(r["us"] / r["ours_us"], 3) if r.get("ours_us") else None
    return rows


def shape_sweep(dev, peaks, with_reference=False):
    """INT4 g128 asymmetric at batch 1 over the six shapes,
    per-case µs and GB/s measured like ``per_case_detail`` (distinct weight
    copies replayed from one graph, more bytes than L2 per replay)."""
    import torch

    from dequant_project_b200.packer import QuantConfig, quantize_tensor

    cs, data = [], []
    for i, (n, k) in enumerate(SHAPE_SWEEP):
        g = torch.Generator(device=dev).manual_seed(7000 + i)
        w = torch.randn(n, k, dtype=torch.float16, device=dev, generator=g) * 0.02
        pw = quantize_tensor(w, QuantConfig(4, 128, False))
        del w
        x = torch.randn(1, k, dtype=torch.float16, device=dev, generator=g)
        cs.append((n, k, 4, 128, False, 1, "int4-g128-asym"))
        data.append((pw, x))
    rows = per_case_detail(dev, cs, data, peaks, min_copies=4)
    if with_reference:
        ref = reference_kernel_detail(dev, cs, data, peaks, rows)
        rows = {"ours": rows, "reference_kernel": ref}
    del data
    torch.cuda.empty_cache()
    return rows


def per_case_detail(dev, cs, data, peaks, reps=20, min_copies=28, gemv_fn=None):
    import torch

    from dequant_project_b200 import dequant_cuda
    gemv = gemv_fn or dequant_cuda.gemv

    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 * 2 ** 20)
    rows = []
    for (n, k, bits, gs, sym, m, name), (pw, x) in zip(cs, data):
        b = case_bytes(n, k, bits, gs, sym, m)
        copies = max(min_copies, math.ceil(8 * l2 / pw.nbytes))
        ws = [(pw.qweight.clone(), pw.scales.clone(),
               None if pw.zeros is None else pw.zeros.clone()) for _ in range(copies)]

        def run():
            for q, s, z in ws:
                gemv(x, q, s, z, bits, gs or k, sym, False)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            run()
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        samples = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            samples.append(e0.elapsed_time(e1) * 1e3 / copies)
        samples.sort()
        us = statistics.median(samples)
        rows.append({"case": f"{n}x{k} {name} M={m}", "bytes": b, "us": round(us, 3),
                     "us_p25": round(samples[len(samples) // 4], 3),
                     "us_p75": round(samples[(3 * len(samples)) // 4], 3),
                     "gb_s": round(b / us * 1e-3, 1),
                     "frac_measured_peak": round(b / us * 1e-3 / peaks["hbm_gbs"], 4),
                     "frac_8tbs": round(b / us * 1e-3 / 8000.0, 4), "copies": copies})
        del g, ws
        torch.cuda.empty_cache()
    return rows


def run_e2e(dev, cs, data, args, dist, local_rank):
    import torch

    from dequant_project_b200 import dequant_cuda

    xs_host = [x.cpu().pin_memory() for _, x in data]
    ys_host = [torch.empty((x.shape[0], pw.qweight.shape[0]), dtype=torch.float16).pin_memory()
               for pw, x in data]
    h2d = sum(x.numel() * 2 for x in xs_host)
    d2h = sum(y.numel() * 2 for y in ys_host)

    def step():
        for i, ((n, k, bits, gs, sym, m, _), (pw, _)) in enumerate(zip(cs, data)):
            xd = xs_host[i].to(dev, non_blocking=True)
            y = dequant_cuda.gemv(xd, pw.qweight, pw.scales, pw.zeros, bits, gs or k, sym, False)
            ys_host[i].copy_(y, non_blocking=True)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_steps = max(1, args.steps // 4)
    e0.record(stream)
    for _ in range(n_steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n_steps
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"ms": ms, "h2d": h2d, "d2h": d2h}


def load_traffic():
    """Per-launch DRAM traffic of the GEMV kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "gemv_dram_traffic.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


# -------------------------------------------------------------- CPU baseline

def cpu_cases_sample(cs, data=None, row_frac=8):
    """The 18 cases restricted to the first N/row_frac rows (the bounded sample).

    With `data` (GPU arm) the packed tensors are copied from the device; without
    (reference arm) the sampled rows are quantized by the numpy oracle.
    """
    import numpy as np

    from oracle import packer_np as P

    out = []
    rng = np.random.default_rng(0)
    for i, (n, k, bits, gs, sym, m, name) in enumerate(cs):
        ns = n // row_frac
        if data is not None:
            pw, x = data[i]
            qw = pw.qweight[:ns].cpu().numpy()
            s = pw.scales[:ns].cpu().numpy()
            z = None if pw.zeros is None else pw.zeros[:ns].cpu().numpy()
            xn = x.cpu().numpy()
        else:
            w = (rng.standard_normal((ns, k)) * 0.02).astype(np.float16)
            qw, s, z = P.quantize_tensor(w, bits, gs, sym, "sequential")
            xn = rng.standard_normal((m, k)).astype(np.float16)
        out.append((ns, k, bits, gs, sym, m, name, xn, qw, s, z))
    return out


def time_cpu_sweep(sample, threads, budget_s):
    from oracle import native

    total_bytes = 0
    passes = 0
    t0 = time.perf_counter()
    while True:
        for (ns, k, bits, gs, sym, m, _, x, qw, s, z) in sample:
            native.gemv(x, qw, s, z, bits, gs or k, sym, False, threads=threads)
            total_bytes += case_bytes(ns, k, bits, gs, sym, m)
        passes += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return total_bytes / el / 1e9, el, passes


def cpu_baseline(cs, data, budget_s=10.0):
    from oracle import native

    sample = cpu_cases_sample(cs, data)
    threads = native.default_threads()
    native.gemv(sample[0][7], *sample[0][8:11], sample[0][2], sample[0][3] or sample[0][1],
                sample[0][4], False, threads=threads)
    gbs, el, passes = time_cpu_sweep(sample, threads, budget_s)
    # The same sample on one thread, as a second row (a short budget).
    gbs1, el1, passes1 = time_cpu_sweep(sample, 1, min(5.0, budget_s))
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"the 18 sweep cases on the first N/8 rows of each weight; {passes} passes "
                      f"in {el:.1f} s; C restatement of F.linear(x, packer.dequantize(pw)), "
                      f"OpenMP, {threads} threads",
            "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                              "sample": f"same sample, {passes1} passes in {el1:.1f} s"}}


DECODE_SAMPLE_ROWS = 8   # rows of each matrix timed = N / DECODE_SAMPLE_ROWS


def _decode_cpu_sample():
    """One Llama-2-7B layer's linears (fused QKV, O, fused gate/up, down) and
    the LM head, INT4 g128 asymmetric, each cut to its first N/8 rows and
    packed by the numpy oracle: (name, rows, k, layers it stands for, x, qw, s, z)."""
    import numpy as np

    from oracle import packer_np as P

    rng = np.random.default_rng(0)
    out = []
    for name, n, k, reps in (("qkv", 12288, 4096, 32), ("o", 4096, 4096, 32),
                             ("gate_up", 22016, 4096, 32), ("down", 4096, 11008, 32),
                             ("lm_head", 32000, 4096, 1)):
        rows = n // DECODE_SAMPLE_ROWS
        w = (rng.standard_normal((rows, k)) * 0.02).astype(np.float16)
        qw, s, z = P.quantize_tensor(w, 4, 128, False, "sequential")
        x = rng.standard_normal((1, k)).astype(np.float16)
        out.append((name, rows, k, reps, x, qw, s, z))
    return out


def _time_decode_cpu(sample, threads):
    """ms per token of the reference CPU path: every sampled GEMV once, scaled
    by rows and by the layers it stands for."""
    from oracle import native

    ms = 0.0
    for (_, rows, k, reps, x, qw, s, z) in sample:
        t0 = time.perf_counter()
        native.gemv(x, qw, s, z, 4, 128, False, False, threads=threads)
        ms += (time.perf_counter() - t0) * 1e3 * DECODE_SAMPLE_ROWS * reps
    return ms


def cpu_decode_baseline(budget_s=10.0):
    """The reference's CPU path (F.linear(x, packer.dequantize(W)) restated in
    C, oracle/cpu_gemv.c) for the headline token, on this host's cores."""
    from oracle import native

    sample = _decode_cpu_sample()
    threads = native.default_threads()
    _time_decode_cpu(sample, threads)
    samples, t0 = [], time.perf_counter()
    while time.perf_counter() - t0 < budget_s or len(samples) < 3:
        samples.append(_time_decode_cpu(sample, threads))
    ms = statistics.median(samples)
    return {"value": round(1000.0 / ms, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "ms_per_token": round(ms, 1),
            "sample": f"one layer's linears (QKV, O, gate/up, down) and the LM head of the "
                      f"headline model, INT4 g128, first N/{DECODE_SAMPLE_ROWS} rows of each, "
                      f"scaled by rows and by 32 layers; attention and norms (<1% of the CPU "
                      f"time) left out; median of {len(samples)} passes in "
                      f"{time.perf_counter() - t0:.1f} s; C restatement of "
                      f"F.linear(x, packer.dequantize(pw)), OpenMP, {threads} threads"}


def run_reference(args, rank, world):
    """The reference CPU path (oracle port) for the headline token, rank 0
    only; other ranks exit 0."""
    if rank != 0:
        return
    from oracle import native

    sample = _decode_cpu_sample()
    threads = native.default_threads()
    for _ in range(max(3, args.warmup)):
        _time_decode_cpu(sample, threads)
    steps = max(3, min(args.steps, 20))
    ms = statistics.median(_time_decode_cpu(sample, threads) for _ in range(steps))
    value = 1000.0 / ms
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp16 activations x int4 codes, fp32 accumulate",
        "data": "synthetic (random-init N(0,0.02) weights)",
        "config": workload_config(world), "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                         "kind": "port",
                         "sample": "each step: one layer's linears and the LM head, first "
                                   f"N/{DECODE_SAMPLE_ROWS} rows of each, scaled to the "
                                   "32-layer token; C restatement of F.linear(x, "
                                   "packer.dequantize(pw)) (oracle/cpu_gemv.c), OpenMP, "
                                   f"{threads} threads"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-detail", action="store_true", help="skip the per-case table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the batch-8 and 70B decoder sub-measurements")
    ap.add_argument("--no-sweep", action="store_true", help="skip the GEMV sweep (N=1)")
    ap.add_argument("--with-70b", action="store_true",
                    help="also run BASELINE config 5 (70B) at N=1")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
