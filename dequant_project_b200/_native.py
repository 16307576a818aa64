"""ctypes binding of libdequant_b200.so, the library's C ABI (include/dequant_b200.h).

The shared library is built in-tree by ``python -m dequant_project_b200.build``.
There is no fallback: if the library is missing or fails to load, every
operation raises, so a GPU run can never silently take a CPU or eager-PyTorch
path.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdequant_b200.so"

_lib = None


class L2Spans(ctypes.Structure):
    """``dqg_l2_spans``: up to 8 device byte ranges to bring into L2."""
    _fields_ = [("ptr", ctypes.c_void_p * 8), ("bytes", ctypes.c_uint64 * 8),
                ("n", ctypes.c_int32)]

    @classmethod
    def of(cls, ranges) -> "L2Spans":
        """From ``(pointer, bytes)`` pairs (at most 8)."""
        ranges = [(p, b) for p, b in ranges if b > 0]
        if len(ranges) > 8:
            raise ValueError(f"at most 8 prefetch ranges, got {len(ranges)}")
        s = cls()
        for i, (p, b) in enumerate(ranges):
            s.ptr[i] = p
            s.bytes[i] = b
        s.n = len(ranges)
        return s


def lib() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built. Build it once with:\n"
            "    python -m dequant_project_b200.build\n"
            "(or call __graft_entry__.build()); re-run after any change under csrc/.")
    h = ctypes.CDLL(str(LIB_PATH))
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    h.dqg_last_error.restype = ctypes.c_char_p
    h.dqg_last_error.argtypes = []
    h.dqg_version.restype = i32
    h.dqg_add_one.restype = i32
    h.dqg_add_one.argtypes = [vp, vp, i64, vp]
    h.dqg_gemv.restype = i32
    h.dqg_gemv.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp]
    h.dqg_gemv_swiglu.restype = i32
    h.dqg_gemv_swiglu.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp]
    h.dqg_gemv_swiglu_supported.restype = i32
    h.dqg_gemv_swiglu_supported.argtypes = [i64, i64, i64, i64, i64, ctypes.POINTER(i32)]
    h.dqg_dequantize.restype = i32
    h.dqg_dequantize.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, vp]
    h.dqg_device_status.restype = i32
    h.dqg_device_status.argtypes = [i32, ctypes.POINTER(ctypes.c_uint32), i32]
    h.dqg_add_rms_norm.restype = i32
    spans = ctypes.POINTER(L2Spans)
    h.dqg_add_rms_norm.argtypes = [vp, vp, vp, vp, i64, i64, ctypes.c_float, spans, vp]
    h.dqg_rope_kv_append.restype = i32
    h.dqg_rope_kv_append.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, spans,
                                     vp]
    h.dqg_silu_mul.restype = i32
    h.dqg_silu_mul.argtypes = [vp, vp, i64, i64, spans, vp]
    h.dqg_set_weight_prefetch.restype = i32
    h.dqg_set_weight_prefetch.argtypes = [i32]
    h.dqg_set_gemv_path.restype = i32
    h.dqg_set_gemv_path.argtypes = [i32]
    h.dqg_debug_gemv_starved.restype = i32
    h.dqg_debug_gemv_starved.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32,
                                         ctypes.c_uint64, vp]
    u64p = ctypes.POINTER(ctypes.c_uint64)
    h.dqg_ipc_export.restype = i32
    h.dqg_ipc_export.argtypes = [vp, vp, u64p]
    h.dqg_ipc_open.restype = i32
    h.dqg_ipc_open.argtypes = [vp, ctypes.POINTER(ctypes.c_void_p)]
    h.dqg_ipc_close.restype = i32
    h.dqg_ipc_close.argtypes = [vp]
    h.dqg_peer_allreduce.restype = i32
    h.dqg_peer_allreduce.argtypes = [vp, vp, i64, u64p, vp, i64, i32, i32, ctypes.c_uint64, vp]
    h.dqg_peer_allreduce_add_rms_norm.restype = i32
    h.dqg_peer_allreduce_add_rms_norm.argtypes = [vp, vp, vp, vp, i64, i64, ctypes.c_float, u64p,
                                                  vp, i64, i32, i32, ctypes.c_uint64, vp]
    h.dqg_gemv_allreduce.restype = i32
    h.dqg_gemv_allreduce.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32,
                                     u64p, u64p, vp, i64, i32, i32, ctypes.c_uint64, vp]
    h.dqg_decode_attention_workspace.restype = i32
    h.dqg_decode_attention_workspace.argtypes = [i64, i64, i64, i64, u64p]
    h.dqg_decode_attention.restype = i32
    h.dqg_decode_attention.argtypes = [vp, vp, vp, vp, vp, ctypes.c_uint64, i64, i64, i64, i64,
                                       i64, i64, vp]
    h.dqg_decode_attention_noalloc.restype = i32
    h.dqg_decode_attention_noalloc.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, vp]
    h.dqg_stream_plan.restype = i32
    h.dqg_stream_plan.argtypes = [i64, i64, i64, i64, i64, i32, ctypes.POINTER(ctypes.c_int32), i32]
    _lib = h
    return _lib


# Every symbol the C header declares; tests check the library exports them all.
EXPORTED = ("dqg_last_error", "dqg_version", "dqg_add_one", "dqg_gemv", "dqg_dequantize",
            "dqg_device_status", "dqg_add_rms_norm", "dqg_rope_kv_append", "dqg_silu_mul",
            "dqg_stream_plan", "dqg_set_weight_prefetch", "dqg_debug_gemv_starved",
            "dqg_set_gemv_path", "dqg_decode_attention_workspace", "dqg_decode_attention",
            "dqg_gemv_allreduce", "dqg_decode_attention_noalloc",
            "dqg_ipc_export", "dqg_ipc_open", "dqg_ipc_close", "dqg_peer_allreduce",
            "dqg_peer_allreduce_add_rms_norm", "dqg_gemv_swiglu",
            "dqg_gemv_swiglu_supported")


def check(rc: int) -> None:
    """Turn a non-zero dqg_status into RuntimeError with the library's message."""
    if rc != 0:
        msg = lib().dqg_last_error().decode(errors="replace")
        raise RuntimeError(msg or f"dequant_b200 call failed with status {rc}")


def device_status(device: int, reset: bool = False) -> int:
    """Read the device-side status word (bit 0: a kernel gave up a bounded wait)."""
    v = ctypes.c_uint32(0)
    check(lib().dqg_device_status(int(device), ctypes.byref(v), int(reset)))
    return v.value
