"""Tensor-parallel sharding of packed linear layers (one process per GPU).

The decode-time linear layers of a decoder shard Megatron-style over the GPUs
of one box:

* column-parallel (QKV, gate, up): each rank holds a contiguous slice of the
  output rows N. No exchange: each rank's output slice feeds its own part of
  the next layer (or is all-gathered).
* row-parallel (O, down): each rank holds a slice of the input dimension K cut
  on quantization-group boundaries, computes a partial product from its slice
  of the activations, and ONE all-reduce (sum, fp16, M x N x 2 bytes) over the
  process group combines the partials; the bias is added once, after it.

Slices are balanced to within one unit and may be uneven: Llama-2-7B's MLP
dimension 11008 is 86 groups of 128, which 8 ranks split as 11,11,11,11,11,
11,10,10 groups. Use the same split for gate/up's N and down's K
(``intermediate_bounds``) so that each rank's SwiGLU output is exactly its
down-projection input.

The packed format is the reference packer's (dequant/packer.py:7-29); a shard
is an ordinary ``PackedWeight`` of the sliced shape, so every kernel and check
of this package applies to it unchanged. The reference has no tensor
parallelism; this follows the sharding its survey describes for the decoder
configurations (hidden sizes split cleanly; the 11008 group rule above).
"""

from __future__ import annotations

from typing import Callable

import torch
from torch import nn

from dequant_project_b200.packer import PackedWeight, QuantConfig


def split_bounds(units: int, world: int) -> list[int]:
    """world + 1 boundaries cutting `units` into balanced contiguous pieces
    (sizes differ by at most one; the larger pieces come first)."""
    if world < 1:
        raise ValueError(f"world size must be >= 1, got {world}")
    if units < world:
        raise ValueError(f"cannot split {units} units over {world} ranks")
    base, extra = divmod(units, world)
    bounds = [0]
    for r in range(world):
        bounds.append(bounds[-1] + base + (1 if r < extra else 0))
    return bounds


def _k_unit(cfg: QuantConfig, k: int) -> int:
    """Smallest K slice the shards of this format can be cut on: one group,
    or for per-channel scales the codes one GEMV lane loads (128 / bits)."""
    if cfg.group_size is None or cfg.group_size >= k:
        return 128 // cfg.bits
    return cfg.group_size


def intermediate_bounds(n_inter: int, cfg: QuantConfig, world: int) -> list[int]:
    """Boundaries (in elements) of the MLP intermediate dimension per rank,
    on the format's K units, shared by gate/up (N) and down (K)."""
    unit = _k_unit(cfg, n_inter)
    if n_inter % unit:
        raise ValueError(f"intermediate size {n_inter} is not a multiple of {unit}")
    return [b * unit for b in split_bounds(n_inter // unit, world)]


def shard_columns(pw: PackedWeight, world: int, rank: int,
                  bounds: list[int] | None = None) -> PackedWeight:
    """Rows [n_lo, n_hi) of the packed weight (column-parallel shard)."""
    n, k = pw.shape
    bounds = bounds or split_bounds(n, world)
    if len(bounds) != world + 1 or bounds[0] != 0 or bounds[-1] != n:
        raise ValueError(f"bad row bounds {bounds} for N={n}, world={world}")
    lo, hi = bounds[rank], bounds[rank + 1]
    return PackedWeight(
        qweight=pw.qweight[lo:hi].contiguous(),
        scales=pw.scales[lo:hi].contiguous(),
        zeros=None if pw.zeros is None else pw.zeros[lo:hi].contiguous(),
        config=pw.config, shape=(hi - lo, k))


def shard_rows(pw: PackedWeight, world: int, rank: int,
               bounds: list[int] | None = None) -> tuple[PackedWeight, int, int]:
    """Input columns [k_lo, k_hi) of the packed weight (row-parallel shard),
    cut on group boundaries. Returns (shard, k_lo, k_hi).

    A per-channel scale applies to a whole row; every shard keeps it, and the
    shard's own per-channel group is its K slice (the partial products are
    linear in the scale, so their sum is the full product)."""
    n, k = pw.shape
    cfg = pw.config
    unit = _k_unit(cfg, k)
    if bounds is None:
        bounds = [b * unit for b in split_bounds(k // unit, world)]
    if len(bounds) != world + 1 or bounds[0] != 0 or bounds[-1] != k:
        raise ValueError(f"bad K bounds {bounds} for K={k}, world={world}")
    if any(b % unit for b in bounds):
        raise ValueError(f"K bounds {bounds} are not multiples of {unit} (group/lane alignment)")
    lo, hi = bounds[rank], bounds[rank + 1]
    pp = cfg.per_pack
    qweight = pw.qweight[:, lo // pp:hi // pp].contiguous()
    per_channel = cfg.group_size is None or cfg.group_size >= k
    if per_channel:
        scales = pw.scales.contiguous()
        zeros = None if pw.zeros is None else pw.zeros.contiguous()
        shard_cfg = QuantConfig(cfg.bits, None, cfg.symmetric, cfg.layout)
    else:
        g = cfg.group_size
        scales = pw.scales[:, lo // g:hi // g].contiguous()
        zeros = None if pw.zeros is None else pw.zeros[:, lo // g:hi // g].contiguous()
        shard_cfg = cfg
    return (PackedWeight(qweight=qweight, scales=scales, zeros=zeros, config=shard_cfg,
                         shape=(n, hi - lo)), lo, hi)


def _default_linear(x: torch.Tensor, pw: PackedWeight) -> torch.Tensor:
    # The fused GEMV for M <= MAX_M, else dequantize + F.linear, as
    # QuantLinear.forward does.
    from dequant_project_b200 import quant_linear as ql
    if x.numel() // pw.shape[1] <= ql.MAX_M:
        return ql.gemv(x, pw)
    return torch.nn.functional.linear(x, ql.dequantize_cuda(pw))


class ColumnParallelQuantLinear(nn.Module):
    """Output rows [n_lo, n_hi) of a packed linear layer on this rank.

    ``forward(x)`` maps the full activations [..., K] to this rank's output
    slice [..., n_hi - n_lo]; with ``gather=True`` it all-gathers the slices
    into the full [..., N] (uneven slices are padded for the collective and
    trimmed after it)."""

    def __init__(self, pw: PackedWeight, world: int, rank: int, bias=None,
                 bounds: list[int] | None = None, group=None, gather: bool = False,
                 linear_fn: Callable | None = None):
        super().__init__()
        n, _ = pw.shape
        self.bounds = bounds or split_bounds(n, world)
        self.world, self.rank, self.group, self.gather = world, rank, group, gather
        self.shard = shard_columns(pw, world, rank, self.bounds)
        lo, hi = self.bounds[rank], self.bounds[rank + 1]
        self.bias = None if bias is None else bias[lo:hi]
        self._linear = linear_fn or _default_linear

    def forward(self, x):
        y = self._linear(x, self.shard)
        if self.bias is not None:
            y = y + self.bias
        if not self.gather or self.world == 1:
            return y
        import torch.distributed as dist
        width = max(b - a for a, b in zip(self.bounds[:-1], self.bounds[1:]))
        lead = y.shape[:-1]
        y2 = y.reshape(-1, y.shape[-1])
        padded = y2.new_zeros((y2.shape[0], width))
        padded[:, :y2.shape[1]] = y2
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded.contiguous(), group=self.group)
        full = torch.cat([p[:, :b - a] for p, a, b in
                          zip(parts, self.bounds[:-1], self.bounds[1:])], dim=1)
        return full.reshape(*lead, full.shape[-1])


class RowParallelQuantLinear(nn.Module):
    """Input columns [k_lo, k_hi) of a packed linear layer on this rank.

    ``forward(x_shard)`` takes this rank's activation slice [..., k_hi - k_lo],
    computes the partial product, sums the partials of all ranks with one
    all-reduce over ``group`` and adds the bias once."""

    def __init__(self, pw: PackedWeight, world: int, rank: int, bias=None,
                 bounds: list[int] | None = None, group=None,
                 linear_fn: Callable | None = None):
        super().__init__()
        self.world, self.rank, self.group = world, rank, group
        self.shard, self.k_lo, self.k_hi = shard_rows(pw, world, rank, bounds)
        self.bias = bias
        self._linear = linear_fn or _default_linear

    def forward(self, x_shard):
        if x_shard.shape[-1] != self.k_hi - self.k_lo:
            raise ValueError(f"rank {self.rank} expects {self.k_hi - self.k_lo} input features, "
                             f"got {x_shard.shape[-1]}")
        y = self._linear(x_shard, self.shard)
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        if self.bias is not None:
            y = y + self.bias
        return y
