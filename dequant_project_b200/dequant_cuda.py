"""Drop-in replacement for the reference's ``dequant_cuda`` torch extension.

Same three functions, same argument names and meaning, same validation and the
same exception type (``RuntimeError``) as KrishnaI2424/Dequant_Project's
binding (kernels/bindings.cpp:5-17, kernels/dequant_cuda.h:10-20):

    add_one(x)
    gemv(x, qweight, scales, zeros, bits, group_size, symmetric, interleaved)
    dequantize(qweight, scales, zeros, bits, group_size, symmetric, interleaved, K)

Each call checks its tensors here (device, dtype, contiguity, shapes -- the
checks of kernels/dequant_gemv.cu:230-283,310-317,339-361), allocates the output
from torch's caching allocator on the input's device, and launches the sm_100a
kernels through the C ABI of libdequant_b200.so on torch's current stream. No
host synchronisation and no host reads of device data, so every call can be
captured in a CUDA graph. There is no CPU path.
"""

from __future__ import annotations

import torch

from dequant_project_b200 import _native

MAX_M = 8


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _on_device:
    """Make `device` current only when it is not already (cheap common case)."""

    def __init__(self, device: torch.device):
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def _check_weight(qweight, scales, zeros, bits, group_size, symmetric, K):
    """check_weight of kernels/dequant_gemv.cu:230-283, same messages."""
    _require(bits in (2, 4, 8), f"bits must be 2, 4 or 8, got {bits}")
    per_pack = 32 // bits
    _require(group_size > 0, f"group_size must be positive, got {group_size}")
    _require(K > 0 and K % group_size == 0,
             f"K={K} is not divisible by group_size={group_size}")
    _require(qweight.is_cuda, "qweight must be a CUDA tensor")
    _require(qweight.dtype == torch.int32, "qweight must be int32")
    _require(qweight.is_contiguous(), "qweight must be contiguous")
    _require(qweight.dim() == 2, f"qweight must be 2-D, got {qweight.dim()}-D")
    _require(qweight.size(1) * per_pack == K,
             f"qweight has {qweight.size(1)} words per row, which is "
             f"{qweight.size(1) * per_pack} codes, but K={K}")
    n = qweight.size(0)
    n_groups = K // group_size
    _require(scales.is_cuda, "scales must be a CUDA tensor")
    _require(scales.dtype == torch.float16, "scales must be float16")
    _require(scales.is_contiguous(), "scales must be contiguous")
    _require(scales.dim() == 2 and scales.size(0) == n and scales.size(1) == n_groups,
             f"scales must be [{n}, {n_groups}], got {list(scales.shape)}")
    _require(scales.device == qweight.device, "scales and qweight must be on the same device")
    _require((zeros is not None) == (not symmetric),
             "symmetric=true takes no zeros" if symmetric else "symmetric=false requires zeros")
    if zeros is not None:
        _require(zeros.is_cuda, "zeros must be a CUDA tensor")
        _require(zeros.dtype == torch.float16, "zeros must be float16")
        _require(zeros.is_contiguous(), "zeros must be contiguous")
        _require(zeros.shape == scales.shape,
                 f"zeros must have the same shape as scales, got {list(zeros.shape)}")
        _require(zeros.device == qweight.device, "zeros and qweight must be on the same device")
    return n


def add_one(x: torch.Tensor) -> torch.Tensor:
    """out = x + 1 for an fp32 CUDA tensor (kernels/smoke.cu:15-25)."""
    _require(x.is_cuda, "x must be a CUDA tensor")
    _require(x.dtype == torch.float32, "x must be float32")
    x = x.contiguous()
    out = torch.empty_like(x)
    with _on_device(x.device):
        _native.check(_native.lib().dqg_add_one(x.data_ptr(), out.data_ptr(), x.numel(),
                                                _stream_handle(x.device)))
    return out


def gemv(x, qweight, scales, zeros, bits, group_size, symmetric, interleaved):
    """y = x @ W^T for a packed W; x fp16 [M, K] with 1 <= M <= 8 -> fp16 [M, N].

    Mirrors kernels/dequant_gemv.cu:339-386 (checks :342-361).
    """
    _require(x.is_cuda, "x must be a CUDA tensor")
    _require(x.dtype == torch.float16, "x must be float16")
    _require(x.is_contiguous(), "x must be contiguous")
    _require(x.dim() == 2, f"x must be 2-D [M, K], got {x.dim()}-D")
    m, k = x.shape
    _require(1 <= m <= MAX_M,
             f"gemv handles 1 <= M <= {MAX_M}, got M={m}; use the dequantize + F.linear fallback")
    _require(x.data_ptr() % 16 == 0, "x must be 16-byte aligned")
    n = _check_weight(qweight, scales, zeros, bits, group_size, symmetric, k)
    _require(x.device == qweight.device, "x and qweight must be on the same device")
    cpl = 128 // bits
    _require(group_size % cpl == 0,
             f"group_size={group_size} must be a multiple of {cpl} (the codes one lane loads "
             f"per uint4) at {bits} bits; this excludes INT2 with group_size 32")
    y = torch.empty((m, n), dtype=torch.float16, device=x.device)
    with _on_device(x.device):
        _native.check(_native.lib().dqg_gemv(
            x.data_ptr(), qweight.data_ptr(), scales.data_ptr(),
            None if zeros is None else zeros.data_ptr(), y.data_ptr(),
            m, n, k, bits, group_size, int(bool(symmetric)), int(bool(interleaved)),
            _stream_handle(x.device)))
    return y


def dequantize(qweight, scales, zeros, bits, group_size, symmetric, interleaved, K):
    """Materialise the packed weight as fp16 [N, K], bit-exact with packer.dequantize.

    Mirrors kernels/dequant_gemv.cu:310-337.
    """
    n = _check_weight(qweight, scales, zeros, bits, group_size, symmetric, K)
    per_pack = 32 // bits
    _require(group_size % per_pack == 0,
             f"group_size={group_size} must be a multiple of {per_pack} values per uint32 "
             f"word at {bits} bits")
    out = torch.empty((n, K), dtype=torch.float16, device=qweight.device)
    with _on_device(qweight.device):
        _native.check(_native.lib().dqg_dequantize(
            qweight.data_ptr(), scales.data_ptr(), None if zeros is None else zeros.data_ptr(),
            out.data_ptr(), n, K, bits, group_size, int(bool(symmetric)),
            int(bool(interleaved)), _stream_handle(qweight.device)))
    return out
