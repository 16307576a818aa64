"""Decode attention as a profiling workload (for ncu and similar tools).

    python tests/profile_attention.py [--batch 1] [--heads 32] [--kv-heads 32]
        [--positions 2049] [--layers 8] [--launches 6]

Builds ``layers`` distinct fp16 KV caches (N(0, 1)) of one sequence batch and
runs ``launches`` attention calls through ``decode_ops.attention`` (the
library's kernel), cycling through the caches so that consecutive launches read
different memory (8 caches of 33.6 MB exceed the 126 MB L2 at the defaults).
The first launches are warm-up; profile the later ones with ``ncu -s``.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> None:
    import torch

    from dequant_project_b200 import decode_ops

    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=32)
    ap.add_argument("--positions", type=int, default=2049)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--launches", type=int, default=6)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    shape = (args.batch, args.kv_heads, args.positions, 128)
    caches = [(torch.randn(shape, generator=g, device=dev).half(),
               torch.randn(shape, generator=g, device=dev).half()) for _ in range(args.layers)]
    q = torch.randn(args.batch, args.heads, 128, generator=g, device=dev).half()
    ws = decode_ops.attention_workspace(args.batch, args.heads, args.kv_heads, args.positions, dev)
    out = None
    for i in range(args.launches):
        kc, vc = caches[i % len(caches)]
        out = decode_ops.attention(q, kc, vc, args.positions, ws)
    torch.cuda.synchronize()
    print(f"ok: {args.launches} launches, batch {args.batch}, {args.heads}/{args.kv_heads} heads, "
          f"{args.positions} positions; out[0,0,:3]={out[0, 0, :3].tolist()}")


if __name__ == "__main__":
    main()
