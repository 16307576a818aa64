"""ctypes loader for the C oracle (TEST INFRASTRUCTURE ONLY).

Wraps ``oracle/cpu_gemv.c`` for numpy arrays. Used by tests/ as a full-size
checker and by bench.py's CPU-baseline leg to time the reference CPU path.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from oracle.build import LIB, build

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        vp, i = ctypes.c_void_p, ctypes.c_int
        _lib.oracle_gemv.argtypes = [vp, i, vp, vp, vp, vp, i, i, i, i, i, i, i]
        _lib.oracle_gemv.restype = i
        _lib.oracle_dequantize.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, i]
        _lib.oracle_dequantize.restype = i
        _lib.oracle_max_threads.restype = i
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def default_threads() -> int:
    return len(os.sched_getaffinity(0))


def gemv(x, qweight, scales, zeros, bits, group_size, symmetric, interleaved, threads=None):
    """fp16 [M,K] x packed [N,K] -> fp16 [M,N] via the C restatement."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    zeros = None if zeros is None else np.ascontiguousarray(zeros, dtype=np.float16)
    m, k = x.shape
    n = qweight.shape[0]
    y = np.empty((m, n), dtype=np.float16)
    rc = lib().oracle_gemv(_ptr(x), m, _ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(y),
                           n, k, bits, group_size, int(symmetric), int(interleaved),
                           threads or default_threads())
    if rc:
        raise ValueError(f"oracle_gemv failed with status {rc}")
    return y


def dequantize(qweight, scales, zeros, bits, group_size, symmetric, interleaved, k, threads=None):
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    zeros = None if zeros is None else np.ascontiguousarray(zeros, dtype=np.float16)
    n = qweight.shape[0]
    out = np.empty((n, k), dtype=np.float16)
    rc = lib().oracle_dequantize(_ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(out), n, k,
                                 bits, group_size, int(symmetric), int(interleaved),
                                 threads or default_threads())
    if rc:
        raise ValueError(f"oracle_dequantize failed with status {rc}")
    return out
