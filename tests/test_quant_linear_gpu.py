"""The Python layer between kernel and model: gemv(), QuantLinear and
quantize_model (scripts/test_quant_linear.py:108-293). References are plain
fp32 PyTorch on the GPU with TF32 and reduced-precision reductions off."""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from dequant_project_b200 import packer
from dequant_project_b200.packer import QuantConfig, quantize_tensor
from dequant_project_b200.quant_linear import (MAX_M, PROJ, QuantLinear, dequantize_cuda, gemv,
                                               quantize_model)

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fp32_reference():
    old = (torch.backends.cuda.matmul.allow_tf32,
           torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    yield
    (torch.backends.cuda.matmul.allow_tf32,
     torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction) = old


def criterion(y, ref, a, depth=1):
    tol = depth * (2 ** -11 * ref.abs() + 2 ** -20 * a)
    ratio = ((y.float() - ref).abs() / (tol + 1e-30)).max().item()
    return ratio <= 1.0, ratio


def exact_weight(pw):
    cfg = pw.config
    n, k = pw.shape
    gs = cfg.effective_group_size(k)
    q = packer.unpack(pw.qweight, cfg, k).reshape(n, k // gs, gs).float()
    off = cfg.bias if cfg.symmetric else pw.zeros.float().unsqueeze(-1)
    return ((q - off) * pw.scales.float().unsqueeze(-1)).reshape(n, k)


def test_constants():
    assert MAX_M == 8
    assert PROJ == ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def test_gemv_reshape_3d():
    torch.manual_seed(0)
    n = k = 3072
    w = torch.randn(n, k, dtype=torch.float16, device="cuda") * 0.02
    pw = quantize_tensor(w, QuantConfig(4, 128, False))
    x = torch.randn(2, 3, k, dtype=torch.float16, device="cuda")
    y = gemv(x, pw)
    assert tuple(y.shape) == (2, 3, n)
    we = exact_weight(pw)
    ok, ratio = criterion(y, F.linear(x.float(), we), F.linear(x.float().abs(), we.abs()))
    assert ok, ratio


@pytest.mark.parametrize("shape", [(1, 3072), (8, 3072), (9, 3072), (64, 3072), (2, 32, 3072)])
def test_quant_linear_both_paths(shape):
    torch.manual_seed(0)
    k, n = 3072, 1024
    lin = nn.Linear(k, n, bias=True).to("cuda", torch.float16)
    ql = QuantLinear.from_linear(lin, QuantConfig(4, 128, False))
    pw = ql._packed()
    assert torch.equal(dequantize_cuda(pw), packer.dequantize(pw))
    x = torch.randn(*shape, dtype=torch.float16, device="cuda")
    y = ql(x)
    m = x.numel() // k
    w_ref = exact_weight(pw) if m <= 8 else packer.dequantize(pw).float()
    ref = F.linear(x.float(), w_ref, ql.bias.float())
    ok, ratio = criterion(y, ref, F.linear(x.float().abs(), w_ref.abs()), depth=2)
    assert ok, (m, ratio)


class _Attn(nn.Module):
    def __init__(self, h):
        super().__init__()
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, name, nn.Linear(h, h, bias=False))


class _Mlp(nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.gate_proj = nn.Linear(h, i, bias=False)
        self.up_proj = nn.Linear(h, i, bias=False)
        self.down_proj = nn.Linear(i, h, bias=False)


class _Block(nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.self_attn = _Attn(h)
        self.mlp = _Mlp(h, i)

    def forward(self, x):
        a = self.self_attn
        x = a.o_proj(a.q_proj(x) + a.k_proj(x) + a.v_proj(x))
        return self.mlp.down_proj(self.mlp.gate_proj(x) + self.mlp.up_proj(x))


class _Fake(nn.Module):
    """Llama's module names with no nonlinearity, so |W|, |x| bound the sums."""

    def __init__(self, h=256, i=512, n_blocks=2):
        super().__init__()
        self.norm = nn.LayerNorm(h)
        self.layers = nn.ModuleList(_Block(h, i) for _ in range(n_blocks))
        self.lm_head = nn.Linear(h, h, bias=False)

    def body(self, h):
        for blk in self.layers:
            h = blk(h)
        return self.lm_head(h)

    def forward(self, x):
        return self.body(self.norm(x))


def test_quantize_model_surgery():
    torch.manual_seed(0)
    h = 256
    model = _Fake(h).to("cuda", torch.float16).eval()
    cfg = QuantConfig(4, 128, False)
    ref_model = copy.deepcopy(model)
    for mod in ref_model.modules():
        if isinstance(mod, nn.Linear) and mod is not ref_model.lm_head:
            mod.weight.data.copy_(packer.dequantize(quantize_tensor(mod.weight.data, cfg)))
    abs_model = copy.deepcopy(ref_model).float()
    for p in abs_model.parameters():
        p.data.abs_()
    stats = quantize_model(model, cfg)
    assert stats["replaced"] == 14
    assert 0 < stats["packed_bytes"] < stats["fp16_bytes"]
    assert isinstance(model.lm_head, nn.Linear) and not isinstance(model.lm_head, QuantLinear)
    assert isinstance(model.norm, nn.LayerNorm)
    assert sum(isinstance(m, QuantLinear) for m in model.modules()) == 14
    x = torch.randn(1, h, dtype=torch.float16, device="cuda")
    with torch.no_grad():
        y = model(x)
        ref = ref_model(x).float()
        a = abs_model.body(ref_model.norm(x).float().abs())
    ok, ratio = criterion(y, ref, a, depth=21)
    assert ok, ratio


def test_quant_linear_graph_capture():
    torch.manual_seed(0)
    k, n = 3072, 1024
    lin = nn.Linear(k, n, bias=True).to("cuda", torch.float16)
    ql = QuantLinear.from_linear(lin, QuantConfig(4, 128, False))
    x = torch.randn(1, k, dtype=torch.float16, device="cuda")
    x2 = torch.randn(1, k, dtype=torch.float16, device="cuda")
    with torch.no_grad():
        eager1 = ql(x).clone()
        eager2 = ql(x2).clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                ql(x)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_y = ql(x)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(static_y, eager1)
        x.copy_(x2)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(static_y, eager2)


def test_module_moves_between_devices():
    lin = nn.Linear(512, 64, bias=False).half()
    ql = QuantLinear.from_linear(lin, QuantConfig(4, 128, True))
    ql = ql.cuda()
    x = torch.randn(1, 512, dtype=torch.float16, device="cuda")
    y = ql(x)
    assert y.device.type == "cuda" and y.shape == (1, 64)
