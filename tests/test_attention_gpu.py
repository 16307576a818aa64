"""Decode attention kernel (dqg_decode_attention) against an fp32 restatement
of softmax(q k^T / sqrt(D)) v on the same fp16 cache: multi-head (the Llama-2-7B
shape) and grouped KV heads (the Llama-3-70B shape), one and many position
splits, ragged lengths, a single position; within 2e-3 of the largest output;
repeated calls bit-identical; the workspace's split counters return to zero (a
second call on the same workspace gives the same bits)."""

from __future__ import annotations

import math

import pytest
import torch

from dequant_project_b200 import _native, decode_ops

pytestmark = pytest.mark.gpu

D = 128


def fp32_attention(q, kc, vc, T):
    m, hq, d = q.shape
    hkv = kc.shape[1]
    g = hq // hkv
    qf = q.float().view(m, hkv, g, d)
    s = torch.einsum("mkgd,mktd->mkgt", qf, kc[:, :, :T].float()) / math.sqrt(d)
    return torch.einsum("mkgt,mktd->mkgd", torch.softmax(s, -1), vc[:, :, :T].float()).reshape(m, hq, d)


CASES = [
    (1, 32, 32, 2049, 2050),     # Llama-2-7B, TP1, batch 1
    (8, 32, 32, 2049, 2049),     # batch 8
    (1, 4, 4, 2049, 2050),       # TP8 shard of the 7B heads
    (1, 64, 8, 4097, 4100),      # Llama-3-70B GQA, TP1
    (8, 8, 1, 4097, 4097),       # 70B TP8 shard, batch 8
    (2, 16, 1, 1, 8),            # a single position
    (3, 6, 2, 65, 70),           # ragged: one position past a tile
    (1, 2, 2, 64, 64),
    (1, 16, 1, 300, 301),        # 16 query heads per KV head
]


@pytest.mark.parametrize("m,hq,hkv,T,cap", CASES, ids=lambda v: str(v))
def test_matches_fp32_restatement(cuda_device, m, hq, hkv, T, cap):
    g = torch.Generator(device=cuda_device).manual_seed(T + hq)
    q = torch.randn(m, hq, D, generator=g, device=cuda_device).half()
    kc = torch.randn(m, hkv, cap, D, generator=g, device=cuda_device).half()
    vc = torch.randn(m, hkv, cap, D, generator=g, device=cuda_device).half()
    ws = decode_ops.attention_workspace(m, hq, hkv, cap, cuda_device)
    out = decode_ops.attention(q, kc, vc, T, ws)
    ref = fp32_attention(q, kc, vc, T)
    err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 2e-3, err
    # A second and third call on the same workspace: only correct if the last
    # CTA of every (sequence, head) reset its split counter.
    for _ in range(2):
        assert torch.equal(decode_ops.attention(q, kc, vc, T, ws), out)
    assert _native.device_status(cuda_device.index) == 0


def test_positions_beyond_T_are_ignored(cuda_device):
    m, hq, hkv, T, cap = 1, 8, 8, 100, 200
    g = torch.Generator(device=cuda_device).manual_seed(1)
    q = torch.randn(m, hq, D, generator=g, device=cuda_device).half()
    kc = torch.randn(m, hkv, cap, D, generator=g, device=cuda_device).half()
    vc = torch.randn(m, hkv, cap, D, generator=g, device=cuda_device).half()
    a = decode_ops.attention(q, kc, vc, T)
    kc[:, :, T:] = 1000.0
    vc[:, :, T:] = float("nan")
    assert torch.equal(decode_ops.attention(q, kc, vc, T), a)


def test_rejects_bad_arguments(cuda_device):
    q = torch.zeros(1, 8, 64, dtype=torch.float16, device=cuda_device)
    kc = torch.zeros(1, 8, 16, 64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="head_dim 128"):
        decode_ops.attention(q, kc, kc, 4, torch.zeros(1 << 20, dtype=torch.uint8,
                                                       device=cuda_device))
    q = torch.zeros(1, 8, D, dtype=torch.float16, device=cuda_device)
    kc = torch.zeros(1, 8, 16, D, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="exceed the cache capacity"):
        decode_ops.attention(q, kc, kc, 17, torch.zeros(1 << 20, dtype=torch.uint8,
                                                        device=cuda_device))
    with pytest.raises(RuntimeError, match="workspace"):
        decode_ops.attention(q, kc, kc, 16, torch.zeros(16, dtype=torch.uint8, device=cuda_device))


def test_one_workspace_serves_every_length(cuda_device):
    """A workspace sized for the capacity, shared by calls of many lengths in
    a row (different numbers of position splits), as the decoder's steps at
    successive positions share it."""
    m, hq, hkv, cap = 1, 32, 32, 2050
    g = torch.Generator(device=cuda_device).manual_seed(9)
    q = torch.randn(m, hq, D, generator=g, device=cuda_device).half()
    kc = torch.randn(m, hkv, cap, D, generator=g, device=cuda_device).half()
    vc = torch.randn(m, hkv, cap, D, generator=g, device=cuda_device).half()
    ws = decode_ops.attention_workspace(m, hq, hkv, cap, cuda_device)
    for T in (1900, 2049, 64, 1, 1000, 2050, 129):
        out = decode_ops.attention(q, kc, vc, T, ws)
        ref = fp32_attention(q, kc, vc, T)
        assert ((out.float() - ref).abs().max() / ref.abs().max()).item() < 2e-3, T
