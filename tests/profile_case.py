"""One GEMV case as a profiling workload (for ncu and similar tools).

    python tests/profile_case.py --n 4096 --k 11008 --bits 4 \
        --group-size 128 --m 1 [--sym] [--copies 8] [--launches 6]

Quantizes `copies` distinct random weights ~N(0, 0.02) of shape [n, k] with
the packer, then launches `launches` GEMVs through the public
``dequant_cuda.gemv`` call, cycling through the copies so that consecutive
launches read different weights (8 copies of a 22 MB matrix exceed the 126 MB
L2). The first `--warm` launches are warm-up; profile the ones after them with
``ncu -s <warm> -c <launches - warm>``.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> None:
    import torch

    from dequant_project_b200 import dequant_cuda
    from dequant_project_b200.packer import QuantConfig, quantize_tensor

    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=11008)
    ap.add_argument("--bits", type=int, default=4, choices=(2, 4, 8))
    ap.add_argument("--group-size", type=int, default=128, help="0 = per-channel (K)")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--sym", action="store_true", help="symmetric quantization")
    ap.add_argument("--interleaved", action="store_true")
    ap.add_argument("--copies", type=int, default=8)
    ap.add_argument("--launches", type=int, default=6)
    ap.add_argument("--warm", type=int, default=3)
    args = ap.parse_args()

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    gs = args.group_size or None
    cfg = QuantConfig(args.bits, gs, args.sym, "interleaved" if args.interleaved else "sequential")
    pws = []
    for _ in range(args.copies):
        w = torch.randn(args.n, args.k, dtype=torch.float16, device=dev) * 0.02
        pws.append(quantize_tensor(w, cfg))
        del w
    x = torch.randn(args.m, args.k, dtype=torch.float16, device=dev)
    torch.cuda.synchronize()
    y = None
    for i in range(args.launches):
        pw = pws[i % len(pws)]
        y = dequant_cuda.gemv(x, pw.qweight, pw.scales, pw.zeros, args.bits, gs or args.k,
                              args.sym, args.interleaved)
    torch.cuda.synchronize()
    print(f"ok: {args.launches} launches of {args.n}x{args.k} int{args.bits} "
          f"g{gs or 'perch'} M={args.m}; y[0,:4]={y[0, :4].tolist()}")


if __name__ == "__main__":
    main()
