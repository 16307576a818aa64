"""Packed low-bit weight format and its offline quantizer (torch, CPU or CUDA).

Public API and bit layout identical to KrishnaI2424/Dequant_Project
``dequant/packer.py`` so that packed tensors move between the two unchanged:

* weights are [N, K]; groups of ``group_size`` consecutive K elements share an
  fp16 scale (and, asymmetric, an fp16 zero-point): scales/zeros [N, K/g];
  ``group_size=None`` is one group per row (packer.py:44-78);
* codes are unsigned; symmetric codes are biased by 2^(bits-1) (packer.py:12-16);
* one int32 word holds 32/bits codes; slot s (bits [b*s, b*s+b)) holds logical
  code s ("sequential") or ``_INTERLEAVE[bits][s]`` ("interleaved")
  (packer.py:18-29,37-41,146-161).

Quantization arithmetic is the reference's, step for step, because the codes
must be bit-identical: the scale is computed in fp32 and rounded to fp16 BEFORE
codes are derived, and rounding is half-to-even (packer.py:99-143).
``pack``/``unpack`` are vectorised (one shift-and-sum over the slot axis
instead of a Python loop over slots).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

# Slot -> logical code order of the interleaved layout (packer.py:37-41). A
# format definition: it must be identical for packed data to be portable.
_INTERLEAVE = {
    4: [0, 2, 4, 6, 1, 3, 5, 7],
    2: [0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15],
    8: [0, 2, 1, 3],
}


@dataclass(frozen=True)
class QuantConfig:
    """Format descriptor (packer.py:44-78)."""

    bits: int = 4
    group_size: int | None = 128   # None means per-channel (one scale per row).
    symmetric: bool = True
    layout: str = "sequential"     # "sequential" | "interleaved"

    def __post_init__(self):
        if self.bits not in (2, 4, 8):
            raise ValueError(f"bits must be 2, 4 or 8, got {self.bits}")
        if self.layout not in ("sequential", "interleaved"):
            raise ValueError(f"unknown layout: {self.layout!r}")
        if self.group_size is not None and self.group_size <= 0:
            raise ValueError("group_size must be positive or None")

    @property
    def per_pack(self):
        """32 / bits: how many codes one int32 word carries."""
        return 32 // self.bits

    @property
    def qmax(self):
        """2^bits - 1, the top of the code range."""
        return (1 << self.bits) - 1

    @property
    def bias(self):
        """2^(bits-1): symmetric codes are stored as q + this, so they fit unsigned."""
        return 1 << (self.bits - 1)

    def groups_for(self, k):
        return 1 if self.group_size is None else k // self.group_size

    def effective_group_size(self, k):
        return k if self.group_size is None else self.group_size


@dataclass
class PackedWeight:
    """Packed codes, per-group scales and (asymmetric) zero-points of one
    [N, K] weight, with its format and shape (packer.py:81-96)."""

    qweight: torch.Tensor          # int32 [N, K // per_pack] (uint32 bit patterns)
    scales: torch.Tensor           # fp16  [N, n_groups]
    zeros: torch.Tensor | None     # fp16  [N, n_groups], asymmetric only
    config: QuantConfig
    shape: tuple                   # original [N, K]

    @property
    def nbytes(self):
        n = self.qweight.numel() * 4 + self.scales.numel() * 2
        if self.zeros is not None:
            n += self.zeros.numel() * 2
        return n


def _slot_order(cfg: QuantConfig):
    return _INTERLEAVE[cfg.bits] if cfg.layout == "interleaved" else list(range(cfg.per_pack))


def quantize(w, cfg: QuantConfig):
    """[N, K] weight -> (int32 codes in [0, qmax], fp16 scales, fp16 zeros or None).

    Same arithmetic as packer.py:99-143.
    """
    if w.dim() != 2:
        raise ValueError(f"expected a 2-D weight, got shape {tuple(w.shape)}")
    n, k = w.shape
    gs = cfg.effective_group_size(k)
    if k % gs:
        raise ValueError(f"K={k} is not divisible by group_size={gs}")
    wf = w.float().reshape(n, k // gs, gs)
    if cfg.symmetric:
        step = wf.abs().amax(dim=-1, keepdim=True) / (cfg.bias - 1)
        zero_point = None
    else:
        hi = wf.amax(dim=-1, keepdim=True)
        lo = wf.amin(dim=-1, keepdim=True)
        step = (hi - lo) / cfg.qmax
    # A zero step (constant group) becomes 1; the step is stored fp16, so the
    # codes are chosen against the fp16 value the kernels will use.
    step = torch.where(step == 0, torch.ones_like(step), step).to(torch.float16).float()
    if cfg.symmetric:
        codes = torch.round(wf / step) + cfg.bias
    else:
        zero_point = torch.round(-lo / step)
        codes = torch.round(wf / step) + zero_point
    codes = codes.clamp_(0, cfg.qmax).to(torch.int32).reshape(n, k)
    scales = step.reshape(n, -1).to(torch.float16)
    zeros = None if zero_point is None else zero_point.reshape(n, -1).to(torch.float16)
    return codes, scales, zeros


def pack(q, cfg: QuantConfig):
    """Unsigned codes [N, K] -> int32 words [N, K // per_pack] (packer.py:146-161)."""
    n, k = q.shape
    per = cfg.per_pack
    if k % per:
        raise ValueError(f"K={k} is not divisible by {per} values per word")
    order = torch.tensor(_slot_order(cfg), device=q.device)
    shifts = torch.arange(per, device=q.device, dtype=torch.int64) * cfg.bits
    slots = q.reshape(n, k // per, per).index_select(-1, order).to(torch.int64) & cfg.qmax
    # Slots occupy disjoint bit ranges, so the sum is the bitwise OR.
    return (slots << shifts).sum(dim=-1).to(torch.int32)


def unpack(packed, cfg: QuantConfig, k):
    """Inverse of pack: int32 words -> unsigned codes [N, K] int32 (packer.py:164-174)."""
    n = packed.shape[0]
    per = cfg.per_pack
    shifts = torch.arange(per, device=packed.device, dtype=torch.int64) * cfg.bits
    words = (packed.to(torch.int64) & 0xFFFFFFFF).reshape(n, k // per, 1)
    slots = ((words >> shifts) & cfg.qmax).to(torch.int32)   # [N, words, per] in slot order
    inverse = torch.empty(per, dtype=torch.int64)
    inverse[torch.tensor(_slot_order(cfg))] = torch.arange(per)
    return slots.index_select(-1, inverse.to(packed.device)).reshape(n, k)


def dequantize(pw: PackedWeight):
    """fp16 [N, K] reconstruction: fp16((q - off) * scale) in fp32 (packer.py:177-189)."""
    cfg = pw.config
    n, k = pw.shape
    gs = cfg.effective_group_size(k)
    q = unpack(pw.qweight, cfg, k).reshape(n, k // gs, gs).float()
    off = cfg.bias if cfg.symmetric else pw.zeros.float().unsqueeze(-1)
    return ((q - off) * pw.scales.float().unsqueeze(-1)).reshape(n, k).to(torch.float16)


def quantize_tensor(w, cfg: QuantConfig) -> PackedWeight:
    """Quantize and pack in one step (packer.py:192-201)."""
    q, scales, zeros = quantize(w, cfg)
    return PackedWeight(qweight=pack(q, cfg), scales=scales, zeros=zeros, config=cfg,
                        shape=tuple(w.shape))
