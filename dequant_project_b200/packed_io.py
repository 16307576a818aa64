"""On-disk format for packed weights.

A file holds named ``PackedWeight``s (the packer's int32 words, fp16 scales and
zero-points, and the format descriptor) plus named plain tensors (an fp16
embedding, say) and a small metadata dict, written with ``torch.save`` and read
back with ``torch.load(weights_only=True)``: nothing but tensors, numbers and
strings is stored, so loading runs no code. Loading a model this way skips
quantization entirely (a 70B-parameter model is packed once, then every rank
reads the file and takes its shard).

The packed layout is the reference packer's (dequant/packer.py:7-29), so a
file's ``qweight/scales/zeros`` are exactly the buffers the reference's
``QuantLinear`` registers (dequant/quant_linear.py:103-106).
"""

from __future__ import annotations

from pathlib import Path

import torch

from dequant_project_b200.packer import PackedWeight, QuantConfig

FORMAT = "dequant_b200.packed"
VERSION = 1


def _record(pw: PackedWeight) -> dict:
    c = pw.config
    return {"qweight": pw.qweight.contiguous(), "scales": pw.scales.contiguous(),
            "zeros": None if pw.zeros is None else pw.zeros.contiguous(),
            "bits": c.bits, "group_size": c.group_size, "symmetric": c.symmetric,
            "layout": c.layout, "shape": list(pw.shape)}


def _packed(name: str, r: dict, device) -> PackedWeight:
    cfg = QuantConfig(int(r["bits"]), None if r["group_size"] is None else int(r["group_size"]),
                      bool(r["symmetric"]), str(r["layout"]))
    n, k = (int(v) for v in r["shape"])
    qw, sc, zr = r["qweight"], r["scales"], r["zeros"]
    groups = cfg.groups_for(k)
    if qw.dtype != torch.int32 or tuple(qw.shape) != (n, k // cfg.per_pack):
        raise ValueError(f"{name}: qweight must be int32 [{n}, {k // cfg.per_pack}], "
                         f"got {qw.dtype} {list(qw.shape)}")
    if sc.dtype != torch.float16 or tuple(sc.shape) != (n, groups):
        raise ValueError(f"{name}: scales must be float16 [{n}, {groups}], got "
                         f"{sc.dtype} {list(sc.shape)}")
    if (zr is None) != cfg.symmetric:
        raise ValueError(f"{name}: zeros must be present exactly when asymmetric")
    if zr is not None and (zr.dtype != torch.float16 or zr.shape != sc.shape):
        raise ValueError(f"{name}: zeros must be float16 like scales")
    mv = (lambda t: t) if device is None else (lambda t: t.to(device))
    return PackedWeight(qweight=mv(qw), scales=mv(sc), zeros=None if zr is None else mv(zr),
                        config=cfg, shape=(n, k))


def save_packed(path, packed: dict[str, PackedWeight], tensors: dict | None = None,
                meta: dict | None = None) -> None:
    """Write named packed weights (and plain tensors, metadata) to ``path``."""
    blob = {"format": FORMAT, "version": VERSION, "meta": dict(meta or {}),
            "packed": {k: _record(v) for k, v in packed.items()},
            "tensors": {k: v.contiguous() for k, v in (tensors or {}).items()}}
    torch.save(blob, Path(path))


def load_packed(path, device=None) -> tuple[dict[str, PackedWeight], dict, dict]:
    """Read a file written by ``save_packed``: (packed weights, tensors, meta),
    moved to ``device`` when given. Raises ValueError for another format or a
    record whose tensors do not match its descriptor."""
    # Memory-mapped: tensors left on the host stay backed by the file, so
    # several processes loading one model share its pages.
    blob = torch.load(Path(path), map_location="cpu", weights_only=True, mmap=True)
    if not isinstance(blob, dict) or blob.get("format") != FORMAT:
        raise ValueError(f"{path} is not a {FORMAT} file")
    if int(blob.get("version", -1)) != VERSION:
        raise ValueError(f"{path}: unsupported version {blob.get('version')}")
    packed = {k: _packed(k, r, device) for k, r in blob["packed"].items()}
    tensors = {k: (v if device is None else v.to(device)) for k, v in blob["tensors"].items()}
    return packed, tensors, blob["meta"]
