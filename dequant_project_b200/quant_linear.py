"""Packed weights behind an ``nn.Linear``-shaped module.

Public surface of KrishnaI2424/Dequant_Project ``dequant/quant_linear.py``
(``MAX_M``, ``PROJ``, ``gemv``, ``dequantize_cuda``, ``QuantLinear`` with
buffers ``qweight/scales/zeros/bias`` and ``from_linear``, ``quantize_model``
returning ``{"replaced", "packed_bytes", "fp16_bytes"}``), served by the B200
kernels of this package. Which kernel runs depends on the number of activation
rows ``M`` (all leading dimensions of ``x`` flattened):

* ``M <= MAX_M``: the fused dequant + GEMV; the weight crosses HBM packed.
* ``M >  MAX_M``: the bit-exact dequantize kernel materialises the fp16 weight
  and ``F.linear`` multiplies (prefill is compute-bound; the reference takes
  the same route, ``quant_linear.py:126-135``).

Nothing here synchronises or reads device data on the host, so modules built
from it can be captured in CUDA graphs. A module keeps the kernel arguments of
its format (bits, group size, symmetry, slot order) from construction on, so a
call costs one binding call and no per-call object construction.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from dequant_project_b200 import dequant_cuda as _ext
from dequant_project_b200.packer import PackedWeight, QuantConfig, quantize_tensor

#: Most activation rows the fused GEMV takes in one call.
MAX_M = _ext.MAX_M

#: Leaf names of the linear layers ``quantize_model`` packs by default: the
#: attention and MLP projections of a Llama-style layer. Embeddings, norms and
#: the LM head are left alone.
PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def _format_args(cfg: QuantConfig, in_features: int) -> tuple:
    """(bits, group_size, symmetric, interleaved) as the kernels take them;
    per-channel formats pass the whole row as one group."""
    return (cfg.bits, cfg.effective_group_size(in_features), bool(cfg.symmetric),
            cfg.layout == "interleaved")


def _rows(x: torch.Tensor, k: int) -> torch.Tensor:
    """``x`` as a contiguous [M, K] matrix."""
    return x.reshape(-1, k).contiguous()


def gemv(x: torch.Tensor, pw: PackedWeight) -> torch.Tensor:
    """``x @ W^T`` for a packed ``W`` [N, K]: ``x`` fp16 [..., K] with at most
    ``MAX_M`` rows in total, result fp16 [..., N]."""
    n, k = pw.shape
    y = _ext.gemv(_rows(x, k), pw.qweight, pw.scales, pw.zeros, *_format_args(pw.config, k))
    return y.view(*x.shape[:-1], n)


def dequantize_cuda(pw: PackedWeight) -> torch.Tensor:
    """The fp16 [N, K] weight rebuilt on the GPU, bit for bit what the packer's
    ``dequantize`` gives."""
    n, k = pw.shape
    return _ext.dequantize(pw.qweight, pw.scales, pw.zeros, *_format_args(pw.config, k), k)


class QuantLinear(nn.Module):
    """A linear layer that holds its weight only as packed codes, fp16 scales
    and (asymmetric formats) fp16 zero-points; ``bias`` is optional fp16."""

    def __init__(self, pw: PackedWeight, bias: torch.Tensor | None = None):
        super().__init__()
        self.out_features, self.in_features = pw.shape
        self.config = pw.config
        self._kargs = _format_args(pw.config, self.in_features)
        # Buffers, so that .to() / .cuda() / state_dict carry them.
        for name, t in (("qweight", pw.qweight), ("scales", pw.scales), ("zeros", pw.zeros),
                        ("bias", bias)):
            self.register_buffer(name, t)

    @classmethod
    def from_linear(cls, linear: nn.Linear, cfg: QuantConfig) -> "QuantLinear":
        """Quantize and pack ``linear``'s weight (on its device) with ``cfg``."""
        bias = linear.bias
        return cls(quantize_tensor(linear.weight.detach(), cfg),
                   None if bias is None else bias.detach().to(torch.float16))

    def _packed(self) -> PackedWeight:
        """The buffers as a ``PackedWeight`` (views, no copies)."""
        return PackedWeight(qweight=self.qweight, scales=self.scales, zeros=self.zeros,
                            config=self.config, shape=(self.out_features, self.in_features))

    def packed_nbytes(self) -> int:
        """Bytes of the packed weight: codes, scales and zero-points."""
        return sum(t.numel() * t.element_size()
                   for t in (self.qweight, self.scales, self.zeros) if t is not None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        k = self.in_features
        x2 = _rows(x, k)
        if x2.shape[0] <= MAX_M:
            y2 = _ext.gemv(x2, self.qweight, self.scales, self.zeros, *self._kargs)
        else:
            w = _ext.dequantize(self.qweight, self.scales, self.zeros, *self._kargs, k)
            y2 = F.linear(x2, w)
        y = y2.view(*x.shape[:-1], self.out_features)
        return y if self.bias is None else y + self.bias

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, config={self.config}")


def quantize_model(model: nn.Module, cfg: QuantConfig, names=PROJ) -> dict:
    """Swap, in place, every ``nn.Linear`` whose attribute name is in ``names``
    for a ``QuantLinear`` packed with ``cfg``; every other module is left as it
    is. Returns how many were swapped and the bytes of their packed and fp16
    weights."""
    wanted = frozenset(names)
    stats = {"replaced": 0, "packed_bytes": 0, "fp16_bytes": 0}
    visited: set[int] = set()

    def visit(parent: nn.Module) -> None:
        if id(parent) in visited:
            return
        visited.add(id(parent))
        for attr, child in list(parent.named_children()):
            if attr in wanted and isinstance(child, nn.Linear):
                q = QuantLinear.from_linear(child, cfg)
                setattr(parent, attr, q)
                stats["replaced"] += 1
                stats["packed_bytes"] += q.packed_nbytes()
                stats["fp16_bytes"] += 2 * child.weight.numel()
            else:
                visit(child)

    visit(model)
    # The replaced fp16 weights are garbage now; hand their blocks back.
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return stats
