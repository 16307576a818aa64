"""The decode-attention entry point that allocates nothing.

``dqg_decode_attention_noalloc`` serves callers that cannot allocate device
memory: its scratch is a static array inside the library instead of a
workspace the caller passes. Through the C ABI, two calls in a row (different
shapes, so the second starts from the first call's leftovers in the shared
array) must match the workspace entry point, ``dqg_decode_attention``, within
the 2e-3 the attention tests use. A call needing more scratch than the array
holds is rejected. This file sorts last so that a run stopping at the first
failure has run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from dequant_project_b200 import _native, decode_ops

pytestmark = pytest.mark.gpu

D = 128


def _noalloc(q, kc, vc, out, T):
    m, hq, d = q.shape
    return _native.lib().dqg_decode_attention_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), m, hq, kc.shape[1], d, T,
        kc.shape[2], torch.cuda.current_stream().cuda_stream)


def _inputs(dev, m, hq, hkv, cap, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(m, hq, D, generator=g, device=dev).half()
    kc = torch.randn(m, hkv, cap, D, generator=g, device=dev).half()
    vc = torch.randn(m, hkv, cap, D, generator=g, device=dev).half()
    return q, kc, vc


def test_matches_the_workspace_entry_point_on_two_calls_in_a_row(cuda_device):
    torch.cuda.set_device(cuda_device)
    calls = [(1, 32, 32, 2049, 2050, 11),   # Llama-2-7B heads, many splits
             (8, 64, 8, 4097, 4097, 12)]    # Llama-3-70B grouped heads, batch 8
    for m, hq, hkv, T, cap, seed in calls:
        q, kc, vc = _inputs(cuda_device, m, hq, hkv, cap, seed)
        out = torch.empty_like(q)
        _native.check(_noalloc(q, kc, vc, out, T))
        ref = decode_ops.attention(q, kc, vc, T,
                                   decode_ops.attention_workspace(m, hq, hkv, cap, cuda_device))
        torch.cuda.synchronize()
        err = ((out.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        assert err < 2e-3, (m, hq, hkv, T, err)
    assert _native.device_status(cuda_device.index) == 0


def test_rejects_a_call_larger_than_the_static_scratch(cuda_device):
    torch.cuda.set_device(cuda_device)
    m, hq, hkv, cap = 64, 64, 64, 4096     # 4096 (sequence, head) pairs: far over 2 MiB
    need = ctypes.c_uint64(0)
    _native.check(_native.lib().dqg_decode_attention_workspace(m, hq, hkv, cap,
                                                               ctypes.byref(need)))
    assert need.value > 2 << 20
    q = torch.zeros(m, hq, D, dtype=torch.float16, device=cuda_device)
    kc = torch.zeros(m, hkv, 16, D, dtype=torch.float16, device=cuda_device)
    rc = _noalloc(q, kc, kc, q, 16)
    assert rc == 2 and b"static scratch" in _native.lib().dqg_last_error()
