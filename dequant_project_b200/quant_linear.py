"""The packed weight as a drop-in ``nn.Linear`` replacement.

Mirrors KrishnaI2424/Dequant_Project ``dequant/quant_linear.py`` (public names
``MAX_M``, ``PROJ``, ``gemv``, ``dequantize_cuda``, ``QuantLinear``,
``quantize_model``; same semantics), backed by the B200 kernels of this
package instead of the reference's extension:

    M <= MAX_M   fused dequant + GEMV (tensor-core MMA over in-register
                 unpacked codes); weights cross HBM packed.
    M >  MAX_M   materialise the fp16 weight with the bit-exact dequantize
                 kernel and call F.linear (cuBLAS), as the reference does
                 (quant_linear.py:126-135).

``forward`` never touches the CPU and never synchronises, so decode steps built
from these modules are CUDA-graph capturable.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from dequant_project_b200 import dequant_cuda as _ext
from dequant_project_b200.packer import PackedWeight, QuantConfig, quantize_tensor

# Largest activation row count the fused GEMV handles (quant_linear.py:38-39).
MAX_M = _ext.MAX_M

# The seven projections per decoder layer that are quantized; norms, embeddings
# and the LM head stay fp16 (quant_linear.py:41-44).
PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def gemv(x, pw: PackedWeight):
    """y = x @ W^T with W held packed. x is [..., K] fp16, y is [..., N] fp16."""
    n, k = pw.shape
    cfg = pw.config
    x2 = x.reshape(-1, k).contiguous()
    y = _ext.gemv(x2, pw.qweight, pw.scales, pw.zeros, cfg.bits, cfg.effective_group_size(k),
                  cfg.symmetric, cfg.layout == "interleaved")
    return y.view(*x.shape[:-1], n)


def dequantize_cuda(pw: PackedWeight):
    """Reconstruct the fp16 [N, K] weight on the GPU, bit-exact with the packer."""
    n, k = pw.shape
    cfg = pw.config
    return _ext.dequantize(pw.qweight, pw.scales, pw.zeros, cfg.bits,
                           cfg.effective_group_size(k), cfg.symmetric,
                           cfg.layout == "interleaved", k)


class QuantLinear(nn.Module):
    """nn.Linear whose weight lives only in packed form (quant_linear.py:96-140)."""

    def __init__(self, pw: PackedWeight, bias=None):
        super().__init__()
        self.out_features, self.in_features = pw.shape
        self.config = pw.config
        self.register_buffer("qweight", pw.qweight)
        self.register_buffer("scales", pw.scales)
        self.register_buffer("zeros", pw.zeros)
        self.register_buffer("bias", bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, cfg: QuantConfig):
        pw = quantize_tensor(linear.weight.data, cfg)
        bias = None if linear.bias is None else linear.bias.data.to(torch.float16)
        return cls(pw, bias)

    def _packed(self):
        # Rebuilt per call so that .to()/.cuda() buffer moves stay correct.
        return PackedWeight(qweight=self.qweight, scales=self.scales, zeros=self.zeros,
                            config=self.config, shape=(self.out_features, self.in_features))

    def forward(self, x):
        pw = self._packed()
        m = x.numel() // self.in_features
        if m <= MAX_M:
            y = gemv(x, pw)
        else:
            y = F.linear(x, dequantize_cuda(pw))
        if self.bias is not None:
            y = y + self.bias
        return y

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, config={self.config}")


def quantize_model(model, cfg: QuantConfig, names=PROJ):
    """Replace every nn.Linear named in `names` with a QuantLinear, in place.

    Returns {"replaced", "packed_bytes", "fp16_bytes"} (quant_linear.py:143-162).
    """
    replaced = 0
    packed_bytes = 0
    fp16_bytes = 0
    for path, mod in list(model.named_modules()):
        leaf = path.rsplit(".", 1)[-1]
        if leaf not in names or not isinstance(mod, nn.Linear):
            continue
        parent = model.get_submodule(path.rsplit(".", 1)[0] if "." in path else "")
        ql = QuantLinear.from_linear(mod, cfg)
        setattr(parent, leaf, ql)
        replaced += 1
        packed_bytes += ql._packed().nbytes
        fp16_bytes += mod.weight.numel() * 2
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return {"replaced": replaced, "packed_bytes": packed_bytes, "fp16_bytes": fp16_bytes}
