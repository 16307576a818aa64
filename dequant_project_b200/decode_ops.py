"""Element-wise steps of the decoder around the packed GEMVs.

CUDA tensors go through the sm_100a kernels of libdequant_b200.so
(``dqg_add_rms_norm``, ``dqg_rope_kv_append``, ``dqg_silu_mul``) on torch's
current stream; if the library is missing these calls raise. CPU tensors take
the same formulas in torch: that branch exists for the host-logic tests of the
tensor-parallel decoder (gloo ranks on the CPU) and is never taken for a CUDA
tensor.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from dequant_project_b200 import _native


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def l2_spans(weights) -> "_native.L2Spans | None":
    """The packed tensors of ``weights`` (PackedWeight objects) as L2 prefetch
    ranges for a decode op, or None when there are none."""
    ranges = []
    for pw in weights:
        for t in (pw.qweight, pw.scales, pw.zeros):
            if t is not None and t.is_cuda:
                ranges.append((t.data_ptr(), t.numel() * t.element_size()))
    return _native.L2Spans.of(ranges) if ranges else None


def _spans_arg(prefetch):
    import ctypes
    return None if prefetch is None else ctypes.byref(prefetch)


def add_rms_norm(h: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor,
                 eps: float, prefetch=None) -> torch.Tensor:
    """If ``delta`` is given, ``h += delta`` in place (fp16); returns
    RMSNorm(h) * weight as fp16 [M, H] (fp32 math). ``prefetch`` (from
    ``l2_spans``) is brought into L2 while the op runs (CUDA only)."""
    if not h.is_cuda:
        if delta is not None:
            h.copy_(h + delta)
        hf = h.float()
        y = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)
        return (y * weight.float()).to(torch.float16)
    m, hd = h.shape
    for t in (h, weight) + (() if delta is None else (delta,)):
        if t.dtype != torch.float16 or not t.is_contiguous():
            raise RuntimeError("add_rms_norm takes contiguous float16 tensors")
    y = torch.empty_like(h)
    _native.check(_native.lib().dqg_add_rms_norm(
        h.data_ptr(), None if delta is None else delta.data_ptr(), weight.data_ptr(),
        y.data_ptr(), m, hd, float(eps), _spans_arg(prefetch), _stream(h)))
    return y


def rope_kv_append(qkv: torch.Tensor, cos_row: torch.Tensor, sin_row: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, pos: int, n_q_heads: int,
                   n_kv_heads: int, prefetch=None) -> torch.Tensor:
    """Rotate the query and key heads of ``qkv`` [M, (Hq + 2 Hkv) D] at one
    position, write keys and values into slot ``pos`` of the caches
    [M, Hkv, capacity, D]; returns the rotated queries [M, Hq, D]."""
    m = qkv.shape[0]
    d = k_cache.shape[-1]
    if not qkv.is_cuda:
        nq, nkv = n_q_heads * d, n_kv_heads * d

        def rot(t):
            tf = t.float()
            h = d // 2
            r = torch.cat([-tf[..., h:], tf[..., :h]], dim=-1)
            return (tf * cos_row + r * sin_row).to(torch.float16)

        q = rot(qkv[:, :nq].reshape(m, n_q_heads, d))
        k_cache[:, :, pos] = rot(qkv[:, nq:nq + nkv].reshape(m, n_kv_heads, d))
        v_cache[:, :, pos] = qkv[:, nq + nkv:].reshape(m, n_kv_heads, d)
        return q
    if not (qkv.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("rope_kv_append takes contiguous tensors")
    if cos_row.dtype != torch.float32 or sin_row.dtype != torch.float32:
        raise RuntimeError("cos/sin rows must be float32")
    q = torch.empty((m, n_q_heads, d), dtype=torch.float16, device=qkv.device)
    _native.check(_native.lib().dqg_rope_kv_append(
        qkv.data_ptr(), cos_row.data_ptr(), sin_row.data_ptr(), q.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), m, n_q_heads, n_kv_heads, d, pos,
        k_cache.shape[2], _spans_arg(prefetch), _stream(qkv)))
    return q


def silu_mul(gate_up: torch.Tensor, prefetch=None) -> torch.Tensor:
    """SwiGLU of ``gate_up`` [M, 2 I] (gate, then up) -> fp16 [M, I]."""
    m, two_i = gate_up.shape
    i = two_i // 2
    if not gate_up.is_cuda:
        return (F.silu(gate_up[:, :i].float()) * gate_up[:, i:].float()).to(torch.float16)
    if not gate_up.is_contiguous() or gate_up.dtype != torch.float16:
        raise RuntimeError("silu_mul takes a contiguous float16 tensor")
    out = torch.empty((m, i), dtype=torch.float16, device=gate_up.device)
    _native.check(_native.lib().dqg_silu_mul(gate_up.data_ptr(), out.data_ptr(), m, i,
                                             _spans_arg(prefetch), _stream(gate_up)))
    return out


def gate_up_order(ir: int) -> torch.Tensor:
    """Row order of a gate/up weight [2 ir, K] (gate rows, then up rows) for
    ``gemv_swiglu``: blocks of 8 gate rows, each followed by the matching 8
    up rows (ir a multiple of 8). Row j of the result is row order[j] of the
    original."""
    if ir % 8:
        raise ValueError(f"the intermediate size {ir} is not a multiple of 8")
    gate = torch.arange(ir // 8)[:, None] * 8 + torch.arange(8)[None, :]
    return torch.cat([gate, gate + ir], dim=1).reshape(-1)


def gemv_swiglu_supported(m: int, n: int, k: int, bits: int, group_size: int) -> bool:
    """Whether ``gemv_swiglu`` has a kernel plan for [m] x [n, k] (CUDA)."""
    import ctypes
    v = ctypes.c_int(0)
    _native.check(_native.lib().dqg_gemv_swiglu_supported(m, n, k, bits, group_size,
                                                          ctypes.byref(v)))
    return bool(v.value)


def gemv_swiglu(x: torch.Tensor, pw) -> torch.Tensor:
    """SwiGLU of the gate/up GEMV in one kernel: ``pw`` is a packed [2 I, K]
    weight in ``gate_up_order``; returns fp16 [M, I] = silu(gate) * up, the
    same values as ``silu_mul`` of the GEMV's de-interleaved output."""
    from dequant_project_b200 import quant_linear as ql
    n, k = pw.shape
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    bits, gs, sym, inter = ql._format_args(pw.config, k)
    out = torch.empty((m, n // 2), dtype=torch.float16, device=x.device)
    _native.check(_native.lib().dqg_gemv_swiglu(
        x2.data_ptr(), pw.qweight.data_ptr(), pw.scales.data_ptr(),
        None if pw.zeros is None else pw.zeros.data_ptr(), out.data_ptr(), m, n, k, bits, gs,
        int(sym), int(inter), _stream(x2)))
    return out


def attention_workspace(m: int, n_q_heads: int, n_kv_heads: int, max_positions: int,
                        device) -> torch.Tensor:
    """Zeroed workspace for ``attention`` calls of up to ``max_positions``
    positions (the library keeps its split counters at zero afterwards)."""
    import ctypes
    n = ctypes.c_uint64(0)
    _native.check(_native.lib().dqg_decode_attention_workspace(
        m, n_q_heads, n_kv_heads, max_positions, ctypes.byref(n)))
    return torch.zeros(max(int(n.value), 16), dtype=torch.uint8, device=device)


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, positions: int,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One query per sequence and head over cache positions 0..positions-1.

    q [M, Hq, D] fp16; k_cache, v_cache [M, Hkv, capacity, D] fp16 (query
    heads grouped consecutively per KV head). Returns [M, Hq, D] fp16. CUDA
    tensors go through ``dqg_decode_attention`` (D = 128; ``workspace`` from
    ``attention_workspace``); CPU tensors take an fp32 softmax(q k^T /
    sqrt(D)) v in torch (the CPU tests' stand-in)."""
    m, hq, d = q.shape
    hkv, cap = k_cache.shape[1], k_cache.shape[2]
    if not q.is_cuda:
        g = hq // hkv
        qf = q.float().view(m, hkv, g, d)
        kc = k_cache[:, :, :positions].float()
        vc = v_cache[:, :, :positions].float()
        s = torch.einsum("mkgd,mktd->mkgt", qf, kc) / math.sqrt(d)
        p = torch.softmax(s, dim=-1)
        return torch.einsum("mkgt,mktd->mkgd", p, vc).reshape(m, hq, d).to(torch.float16)
    for t in (q, k_cache, v_cache):
        if t.dtype != torch.float16 or not t.is_contiguous():
            raise RuntimeError("attention takes contiguous float16 tensors")
    if workspace is None:
        workspace = attention_workspace(m, hq, hkv, positions, q.device)
    out = torch.empty_like(q)
    _native.check(_native.lib().dqg_decode_attention(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
        workspace.data_ptr(), workspace.numel(), m, hq, hkv, d, positions, cap, _stream(q)))
    return out
