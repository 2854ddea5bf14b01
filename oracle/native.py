"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): ctypes binding of the C + OpenMP oracle (oracle/c/oracle.c)."""

import ctypes
import os

import numpy as np

from . import build as _build

_lib = None
P = ctypes.c_void_p
I64 = ctypes.c_int64


def load():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        lib = ctypes.CDLL(path)
        lib.orc_quant_q8_0.argtypes = [P, I64, I64, P, P]
        lib.orc_quant_q8_K.argtypes = [P, I64, I64, P, P, P]
        lib.orc_gemv.argtypes = [ctypes.c_int, P, I64, P, P, P, I64, I64, I64, P, P, ctypes.c_int]
        lib.orc_max_threads.restype = ctypes.c_int
        lib.orc_set_threads.argtypes = [ctypes.c_int]
        # one thread per core this process may use, whatever OMP_NUM_THREADS says (torchrun sets it to 1)
        lib.orc_set_threads(len(os.sched_getaffinity(0)))
        lib.orc_half_to_float.argtypes = [ctypes.c_uint16]
        lib.orc_half_to_float.restype = ctypes.c_float
        lib.orc_float_to_half.argtypes = [ctypes.c_float]
        lib.orc_float_to_half.restype = ctypes.c_uint16
        _lib = lib
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def quant_q8_0(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    xq = np.empty((m, k), np.int8)
    xd = np.empty((m, k // 32), np.float32)
    load().orc_quant_q8_0(_p(x), m, k, _p(xq), _p(xd))
    return xq, xd


def quant_q8_K(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    xq = np.empty((m, k), np.int8)
    xd = np.empty((m, k // 256), np.float32)
    bs = np.empty((m, k // 256, 16), np.int16)
    load().orc_quant_q8_K(_p(x), m, k, _p(xq), _p(xd), _p(bs))
    return xq, xd, bs


def gemv(fmt, wq, ws, xq, xd, k, want_s=False, threads=0):
    """-> (reference f64 [M][N], int32 block dots [M][N][nb] or None)."""
    wq = np.ascontiguousarray(wq, dtype=np.uint8)
    ws = np.ascontiguousarray(ws, dtype=np.int16)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    xd = np.ascontiguousarray(xd, dtype=np.float32)
    n, m = wq.shape[0], xq.shape[0]
    nb = k // (256 if fmt in ("tq2_0", "q4_k") else 32)
    y = np.empty((m, n), np.float64)
    s = np.empty((m, n, nb), np.int32) if want_s else None
    load().orc_gemv({"q4_0": 0, "tq2_0": 1, "q8_0": 2, "iq4_nl": 3, "q4_k": 4}[fmt], _p(wq), wq.shape[1], _p(ws), _p(xq), _p(xd), n, k, m, _p(y),
                    _p(s) if want_s else None, threads)
    return y, s


def max_threads():
    return int(load().orc_max_threads())
