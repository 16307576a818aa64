#!/usr/bin/env python
"""Benchmark of the fused low-bit dequant + GEMV path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the bit-width sweep): GEMV with W 4096x11008 and
11008x4096, quantized INT8 per-channel symmetric, INT4 group-128 asymmetric
and INT2 group-64 asymmetric, activations x fp16 [M, K] for M = 1, 4, 8 -- 18
cases. Weights are random-init ~N(0, 0.02) quantized by the product packer,
activations ~N(0, 1) (synthetic; the reference has no dataset). Every case has
its own packed tensors, so one step touches ~480 MB of distinct weights, far
more than the 126 MB L2: no case is served from L2.

One step = the 18 GEMVs once, replayed from one CUDA graph. ``value`` is the
whole-job achieved HBM bandwidth, algorithmic bytes (byte_model.gemv_bytes)
over device time, summed over ranks (each rank runs its own sweep: weak
scaling, no collective on the data path). ``e2e`` is the same metric through
the public ``dequant_cuda.gemv`` call with the activations copied from pinned
host memory and the outputs copied back inside the timed region.

``shape_sweep`` (one GPU) is BASELINE config 3: INT4 g128 at batch 1 over
(4096,4096), (12288,4096), (4096,14336), (28672,8192), (8192,28672) and
(128256,4096), per case µs and GB/s.

``decode`` adds decode ms/token of the tensor-parallel decoder at TP = N
(Llama-2-7B architecture, every linear and the LM head INT4
g128 packed, batch 1, 2048-token fp16 KV cache), from a CUDA graph of one step,
max over ranks (dequant_project_b200/decode_bench.py).

``--impl reference`` times the reference's CPU path (the C restatement of
``F.linear(x, packer.dequantize(pw))`` in oracle/, all host threads) on a
bounded row sample of the same 18 cases, on rank 0 only.
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

METRIC = ("GEMV achieved HBM GB/s over the bit-width sweep "
          "(INT8 per-ch / INT4 g128 / INT2 g64; 4096x11008 & 11008x4096; M=1,4,8)")
UNIT = "GB/s"
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
    return {"workload": "bit-width sweep (BASELINE config 2): 18 GEMVs/step",
            "shapes": ["4096x11008", "11008x4096"],
            "formats": [f[3] for f in FORMATS], "batches": list(BATCHES),
            "l2": "inputs > L2 (18 distinct packed matrices, ~480 MB per step)",
            "parallelism": f"replicas x{world} (weak)"}


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

def run_ours(args, rank, world, local_rank):
    import torch

    from dequant_project_b200 import dequant_cuda
    from dequant_project_b200.byte_model import measured_peaks
    from dequant_project_b200.packer import QuantConfig, quantize_tensor

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    cs = cases()
    # Weights: one distinct packed matrix per case (so M=1/4/8 do not share L2).
    data = []
    for i, (n, k, bits, gs, sym, m, _) in enumerate(cs):
        g = torch.Generator(device=dev).manual_seed(1000 * rank + i)
        w = torch.randn(n, k, dtype=torch.float16, device=dev, generator=g) * 0.02
        pw = quantize_tensor(w, QuantConfig(bits, gs, sym))
        del w
        x = torch.randn(m, k, dtype=torch.float16, device=dev, generator=g)
        data.append((pw, x))
    torch.cuda.synchronize()
    step_bytes = sum(case_bytes(n, k, bits, gs, sym, m) for (n, k, bits, gs, sym, m, _) in cs)

    def step():
        ys = []
        for (n, k, bits, gs, sym, m, _), (pw, x) in zip(cs, data):
            ys.append(dequant_cuda.gemv(x, pw.qweight, pw.scales, pw.zeros, bits, gs or k, sym,
                                        False))
        return ys

    # Capture one step in a CUDA graph (side-stream warm-up first).
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_ys = step()
    del static_ys

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])

    # Warm-up, including ~1 s of replays so that clocks are settled when the
    # timed region starts; clocks are sampled throughout.
    with ClockSampler(local_rank) as clk:
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize()
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < 1.0:
            for _ in range(50):
                graph.replay()
            torch.cuda.synchronize()
        stream = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clocks = clk.summary(t0 - 1.2, t1)

    value = step_bytes * world / (ms * 1e-3) / 1e9
    peaks = measured_peaks()
    per_gpu = step_bytes / (ms * 1e-3) / 1e9

    # Per-case µs (the reference's method: n_copies distinct weights replayed
    # in one graph, scripts/bench_dequant_kernel.py:119-168), rank 0, 1 GPU.
    detail = None
    if rank == 0 and world == 1 and not args.no_detail:
        detail = per_case_detail(dev, cs, data, peaks)
    shapes = None
    if rank == 0 and world == 1 and not args.no_detail:
        try:
            shapes = shape_sweep(dev, peaks)
        except Exception as exc:  # noqa: BLE001 - reported, never fatal to the line
            shapes = {"error": f"{type(exc).__name__}: {exc}"[:300]}

    # End to end through the public API with host buffers.
    e2e = run_e2e(dev, cs, data, args, dist, local_rank)
    e2e_value = step_bytes * world / (e2e["ms"] * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cs, data, budget_s=args.cpu_seconds)

    # Decode ms/token of the tensor-parallel decoder at TP = world (BASELINE
    # config 4: Llama-2-7B architecture, INT4 g128, batch 1, 2048-token KV
    # cache), timed the same way (CUDA events, max over ranks). A failure here
    # is reported in the line and never voids the GEMV result.
    decode = None
    if not args.no_decode:
        try:
            from dequant_project_b200 import decode_bench
            decode = decode_bench.measure(decode_bench.default_args(), dist, rank, world, dev)
        except Exception as exc:  # noqa: BLE001
            decode = {"error": f"{type(exc).__name__}: {exc}"[:300]}

    traffic = load_traffic()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 activations x int2/4/8 codes, fp32 accumulate",
            "data": "synthetic (random-init N(0,0.02) weights, N(0,1) activations)",
            "config": workload_config(world),
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 2),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(per_gpu / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, copy)",
                         "kernel": "dqg::stream::gemv_stream_kernel (all 18 launches of a step)",
                         "bytes_per_launch_avg": step_bytes // len(cs),
                         "traffic": traffic},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "ms_per_step": round(e2e["ms"], 4),
                    "path": "dequant_cuda.gemv (eager, pinned host x -> device -> pinned host y)"},
            "gpu_launches": len(cs) * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "detail": detail,
            "decode": decode,
            "shape_sweep": shapes,
        }
        print(json.dumps(line), flush=True)
    del graph
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


SHAPE_SWEEP = [(4096, 4096), (12288, 4096), (4096, 14336), (28672, 8192), (8192, 28672),
               (128256, 4096)]


def shape_sweep(dev, peaks):
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
    del data
    torch.cuda.empty_cache()
    return rows


def per_case_detail(dev, cs, data, peaks, reps=20, min_copies=28):
    import torch

    from dequant_project_b200 import dequant_cuda

    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 * 2 ** 20)
    rows = []
    for (n, k, bits, gs, sym, m, name), (pw, x) in zip(cs, data):
        b = case_bytes(n, k, bits, gs, sym, m)
        copies = max(min_copies, math.ceil(8 * l2 / pw.nbytes))
        ws = [(pw.qweight.clone(), pw.scales.clone(),
               None if pw.zeros is None else pw.zeros.clone()) for _ in range(copies)]

        def run():
            for q, s, z in ws:
                dequant_cuda.gemv(x, q, s, z, bits, gs or k, sym, False)

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
    return {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"the 18 sweep cases on the first N/8 rows of each weight; {passes} passes "
                      f"in {el:.1f} s; C restatement of F.linear(x, packer.dequantize(pw)), "
                      f"OpenMP, {threads} threads",
            "single_thread": {"value": round(gbs1, 3), "unit": UNIT, "cores": 1,
                              "sample": f"same sample, {passes1} passes in {el1:.1f} s"}}


def run_reference(args, rank, world):
    """The reference CPU path (oracle port), rank 0 only; other ranks exit 0."""
    if rank != 0:
        return
    from oracle import native

    cs = cases()
    sample = cpu_cases_sample(cs, None)
    threads = native.default_threads()
    from oracle import native as _n
    _n.lib()
    step_bytes = sum(case_bytes(ns, k, bits, gs, sym, m)
                     for (ns, k, bits, gs, sym, m, *_r) in sample)

    def step():
        for (ns, k, bits, gs, sym, m, _, x, qw, s, z) in sample:
            native.gemv(x, qw, s, z, bits, gs or k, sym, False, threads=threads)

    for _ in range(max(3, args.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    ms = el / args.steps * 1e3
    value = step_bytes / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 activations x int2/4/8 codes, fp32 accumulate",
        "data": "synthetic (random-init N(0,0.02) weights, N(0,1) activations)",
        "config": workload_config(1), "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads,
                         "kind": "port",
                         "sample": "each step: the 18 sweep cases on the first N/8 rows of each "
                                   "weight; C restatement of F.linear(x, packer.dequantize(pw)) "
                                   f"(oracle/cpu_gemv.c), OpenMP, {threads} threads"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-detail", action="store_true", help="skip the per-case table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the decoder ms/token measurement")
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
