"""Generate the golden vectors that pin the oracle to the reference.

Run once, in a container where the reference project is mounted:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py REFERENCE_ROOT

(REFERENCE_ROOT, or the environment variable DEQUANT_REFERENCE_ROOT: the
checkout of the reference project.)

It imports the reference's own packer (``dequant/packer.py`` of
KrishnaI2424/Dequant_Project, read-only) and its CPU GEMV path
``F.linear(x, packer.dequantize(pw))`` and writes:

  packer_cases.json  sha256 prefixes of qweight / scales / zeros / dequantized
                     weight for every bits x layout x symmetry x group format on
                     seeded 64x512 inputs (Gaussian, and skewed for asymmetric),
                     plus the reference's M=1..8 GEMV outputs as hex fp16;
  known_answers.json the same hashes (and y) at the benchmark shapes.

Input recipe (identical in the tests that consume these files): CPU generator,
``torch.manual_seed(seed)``; then ``gauss = randn(N, K, fp16) * 0.02``,
``skew = (rand(N, K) * 0.5 + 2.0).to(fp16)``, ``x = randn(8, K, fp16)`` drawn in
that order.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
BITS = (2, 4, 8)
LAYOUTS = ("sequential", "interleaved")
GROUPS = (32, 64, 128, 256, None)


def h(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()[:16]


def small_inputs(seed: int, n: int = 64, k: int = 512):
    torch.manual_seed(seed)
    gauss = torch.randn(n, k, dtype=torch.float16) * 0.02
    skew = (torch.rand(n, k) * 0.5 + 2.0).to(torch.float16)
    x = torch.randn(8, k, dtype=torch.float16)
    return gauss, skew, x


def main(ref_root: str) -> None:
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    from dequant import packer  # the reference's own module

    src = Path(ref_root, "dequant", "packer.py").read_bytes()
    meta = {"reference_packer_sha256": hashlib.sha256(src).hexdigest(),
            "torch": torch.__version__}

    torch.set_num_threads(1)
    gauss, skew, x = small_inputs(0)
    cases = []
    for bits in BITS:
        for layout in LAYOUTS:
            for sym in (True, False):
                for gs in GROUPS:
                    inputs = [("gauss", gauss)] if sym else [("gauss", gauss), ("skew", skew)]
                    for tag, w in inputs:
                        cfg = packer.QuantConfig(bits, gs, sym, layout)
                        pw = packer.quantize_tensor(w, cfg)
                        deq = packer.dequantize(pw)
                        case = {
                            "bits": bits, "group_size": gs, "symmetric": sym,
                            "layout": layout, "input": tag, "N": 64, "K": 512,
                            "qweight": h(pw.qweight), "scales": h(pw.scales),
                            "zeros": None if pw.zeros is None else h(pw.zeros),
                            "deq": h(deq),
                        }
                        if tag == "gauss":
                            y = F.linear(x, deq)  # reference CPU GEMV path, M=8
                            case["y_fp16_hex"] = y.contiguous().view(torch.int16).numpy() \
                                .astype("<u2").tobytes().hex()
                        cases.append(case)
    (HERE / "packer_cases.json").write_text(json.dumps({"meta": meta, "cases": cases}, indent=1))

    torch.set_num_threads(8)
    big = []
    for (n, k), formats in [
        ((4096, 4096), [(4, 128, False)]),
        ((4096, 11008), [(8, None, True), (4, 128, False), (2, 64, False)]),
        ((11008, 4096), [(8, None, True), (4, 128, False), (2, 64, False)]),
    ]:
        torch.manual_seed(0)
        w = torch.randn(n, k, dtype=torch.float16) * 0.02
        xv = torch.randn(1, k, dtype=torch.float16)
        for bits, gs, sym in formats:
            cfg = packer.QuantConfig(bits, gs, sym)
            pw = packer.quantize_tensor(w, cfg)
            y = F.linear(xv, packer.dequantize(pw))
            big.append({"N": n, "K": k, "bits": bits, "group_size": gs, "symmetric": sym,
                        "layout": "sequential", "w": h(w), "qweight": h(pw.qweight),
                        "scales": h(pw.scales),
                        "zeros": None if pw.zeros is None else h(pw.zeros),
                        "y": h(y),
                        "y_fp16_hex": y.contiguous().view(torch.int16).numpy()
                        .astype("<u2").tobytes().hex()})
    (HERE / "known_answers.json").write_text(json.dumps({"meta": meta, "cases": big}, indent=1))
    print(f"{len(cases)} small cases, {len(big)} benchmark-shape cases")


if __name__ == "__main__":
    import os
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DEQUANT_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (the reference project's checkout)")
    main(root)
