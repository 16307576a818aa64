"""numpy restatement of the reference packer and its CPU GEMV path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the product never imports
this module.

Every function follows one function of the reference project
(KrishnaI2424/Dequant_Project) and cites it. Arithmetic is done in the same
precision and in the same order as the reference's torch code so that the
integer and fp16 outputs are bit-identical:

* scales are computed in fp32 and rounded to fp16 BEFORE codes are derived
  (``dequant/packer.py:119-125,135``);
* ``round`` is round-half-to-even (``torch.round`` == ``np.rint``);
* dequantization is ``fp16((q - off) * scale)`` with both operations in fp32
  (``dequant/packer.py:177-189``).
"""

from __future__ import annotations

import numpy as np

# Slot -> logical code order inside one 32-bit word for the "interleaved"
# layout (dequant/packer.py:37-41). Slot s of a word holds logical code
# INTERLEAVE[bits][s] of that word's group of 32/bits codes.
INTERLEAVE = {
    4: (0, 2, 4, 6, 1, 3, 5, 7),
    2: (0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15),
    8: (0, 2, 1, 3),
}


def fmt_params(bits: int):
    """(per_pack, qmax, bias) of a bit width (dequant/packer.py:59-72)."""
    if bits not in (2, 4, 8):
        raise ValueError(f"bits must be 2, 4 or 8, got {bits}")
    return 32 // bits, (1 << bits) - 1, 1 << (bits - 1)


def slot_order(bits: int, layout: str):
    """Logical index held by each slot of a word (dequant/packer.py:152,168)."""
    per = 32 // bits
    if layout == "interleaved":
        return INTERLEAVE[bits]
    if layout == "sequential":
        return tuple(range(per))
    raise ValueError(f"unknown layout: {layout!r}")


def effective_group(k: int, group_size):
    """group_size None means one group per row (dequant/packer.py:77-78)."""
    return k if group_size is None else group_size


def quantize(w: np.ndarray, bits: int, group_size, symmetric: bool):
    """Restates ``quantize`` (dequant/packer.py:99-143).

    w is fp16 [N, K]. Returns (codes int32 [N, K], scales fp16 [N, G],
    zeros fp16 [N, G] or None).
    """
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight, got shape {w.shape}")
    _, qmax, bias = fmt_params(bits)
    n, k = w.shape
    gs = effective_group(k, group_size)
    if k % gs:
        raise ValueError(f"K={k} is not divisible by group_size={gs}")
    one = np.float32(1.0)
    wf = w.astype(np.float32).reshape(n, k // gs, gs)
    if symmetric:
        amax = np.abs(wf).max(axis=-1, keepdims=True)
        scales = amax / np.float32(bias - 1)
        scales = np.where(scales == 0, one, scales).astype(np.float32)
        scales = scales.astype(np.float16).astype(np.float32)
        q = np.rint(wf / scales) + np.float32(bias)
        zeros = None
    else:
        wmax = wf.max(axis=-1, keepdims=True)
        wmin = wf.min(axis=-1, keepdims=True)
        scales = (wmax - wmin) / np.float32(qmax)
        scales = np.where(scales == 0, one, scales).astype(np.float32)
        scales = scales.astype(np.float16).astype(np.float32)
        zeros = np.rint(-wmin / scales)
        q = np.rint(wf / scales) + zeros
    q = np.clip(q, 0, qmax).astype(np.int32).reshape(n, k)
    scales = scales.reshape(n, -1).astype(np.float16)
    if zeros is not None:
        zeros = zeros.reshape(n, -1).astype(np.float16)
    return q, scales, zeros


def pack(q: np.ndarray, bits: int, layout: str) -> np.ndarray:
    """Restates ``pack`` (dequant/packer.py:146-161): codes -> int32 words."""
    per, qmax, _ = fmt_params(bits)
    n, k = q.shape
    if k % per:
        raise ValueError(f"K={k} is not divisible by {per} values per word")
    blocks = q.reshape(n, k // per, per).astype(np.int64)
    out = np.zeros((n, k // per), dtype=np.int64)
    for slot, logical in enumerate(slot_order(bits, layout)):
        out |= (blocks[:, :, logical] & qmax) << (bits * slot)
    return out.astype(np.int32)  # wraps to the uint32 bit pattern


def unpack(packed: np.ndarray, bits: int, layout: str, k: int) -> np.ndarray:
    """Restates ``unpack`` (dequant/packer.py:164-174): words -> codes int32."""
    per, qmax, _ = fmt_params(bits)
    n = packed.shape[0]
    words = packed.astype(np.int64) & 0xFFFFFFFF
    out = np.zeros((n, k // per, per), dtype=np.int32)
    for slot, logical in enumerate(slot_order(bits, layout)):
        out[:, :, logical] = ((words >> (bits * slot)) & qmax).astype(np.int32)
    return out.reshape(n, k)


def dequantize(qweight, scales, zeros, bits, group_size, symmetric, layout, k):
    """Restates ``dequantize`` (dequant/packer.py:177-189) -> fp16 [N, K]."""
    _, _, bias = fmt_params(bits)
    n = qweight.shape[0]
    gs = effective_group(k, group_size)
    q = unpack(qweight, bits, layout, k).reshape(n, k // gs, gs).astype(np.float32)
    s = scales.astype(np.float32)[:, :, None]
    if symmetric:
        w = (q - np.float32(bias)) * s
    else:
        w = (q - zeros.astype(np.float32)[:, :, None]) * s
    return w.reshape(n, k).astype(np.float16)


def exact_weight(qweight, scales, zeros, bits, group_size, symmetric, layout, k):
    """(code - offset) * scale in fp32 WITHOUT the fp16 store.

    Restates ``exact_weight`` of the reference kernel gate
    (scripts/test_dequant_kernel.py:92-109): the weight a register-only GEMV
    actually multiplies by.
    """
    _, _, bias = fmt_params(bits)
    n = qweight.shape[0]
    gs = effective_group(k, group_size)
    q = unpack(qweight, bits, layout, k).reshape(n, k // gs, gs).astype(np.float32)
    off = np.float32(bias) if symmetric else zeros.astype(np.float32)[:, :, None]
    return ((q - off) * scales.astype(np.float32)[:, :, None]).reshape(n, k)


def quantize_tensor(w, bits, group_size, symmetric, layout):
    """Restates ``quantize_tensor`` (dequant/packer.py:192-201)."""
    q, scales, zeros = quantize(w, bits, group_size, symmetric)
    return pack(q, bits, layout), scales, zeros


def gemv_ref(x, qweight, scales, zeros, bits, group_size, symmetric, layout):
    """The reference CPU GEMV path ``F.linear(x, packer.dequantize(pw))``.

    x fp16 [M, K] -> fp16 [M, N]: fp16 weights from ``dequantize``, products and
    sums in fp32, one rounding to fp16 at the end (the way torch's CPU
    ``F.linear`` treats fp16 operands). Summation order differs from torch's, so
    this agrees with the reference to fp32 rounding, not bit for bit.
    """
    k = x.shape[1]
    wd = dequantize(qweight, scales, zeros, bits, group_size, symmetric, layout, k)
    return (x.astype(np.float32) @ wd.astype(np.float32).T).astype(np.float16)


def gemv_criterion(y, ref, absw, absx):
    """Elementwise error and tolerance of the reference kernel gate.

    ``|y - ref| <= 2^-11 |ref| + 2^-20 (|W| @ |x|^T)``
    (scripts/test_dequant_kernel.py:112-122). ref is fp32 [M, N]; absw [N, K]
    and absx [M, K] are fp32 magnitudes. Returns (err, tol), both [M, N].
    """
    a = absx.astype(np.float64) @ absw.astype(np.float64).T
    tol = 2.0 ** -11 * np.abs(ref.astype(np.float64)) + 2.0 ** -20 * a
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    return err, tol


def max_rel_err(y, ref) -> float:
    """max|y - ref| / max|ref|: the 2e-3 acceptance metric of the GEMV path."""
    ref = ref.astype(np.float64)
    d = np.abs(y.astype(np.float64) - ref).max()
    m = np.abs(ref).max()
    return float(d / m) if m > 0 else float(d)
