"""ctypes binding of the C-ABI library `libcompb200.so` (declarations: include/comp_b200.h).

The library is loaded from this package directory only (built in-tree by `comp_b200.build`). There is no fallback:
if it is missing, every compute entry point raises.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcompb200.so")

B2Q_OK = 0
ERRORS = {-1: "EINVAL", -2: "EALIGN", -3: "ECUDA", -4: "ERANGE", -5: "ETIMEOUT"}

P = ctypes.c_void_p
I64 = ctypes.c_int64
INT = ctypes.c_int

# name -> (restype, argtypes); every symbol include/comp_b200.h declares
SIGNATURES = {
    "b2q_version": (ctypes.c_char_p, []),
    "b2q_last_error": (INT, [ctypes.c_char_p, ctypes.c_size_t]),
    "b2q_launch_count": (ctypes.c_longlong, []),
    "b2q_quant_q8_0": (INT, [P, I64, P, P, I64, I64, P]),
    "b2q_quant_q8_K": (INT, [P, I64, P, P, P, I64, I64, P]),
    "b2q_gemv_q4_0": (INT, [P, I64, P, P, P, P, P, I64, I64, I64, INT, P]),
    "b2q_gemv_tq2_0": (INT, [P, I64, P, P, P, P, P, I64, I64, I64, INT, P]),
    "b2q_gemv_q8_0": (INT, [P, I64, P, P, P, P, P, I64, I64, I64, INT, P]),
    "b2q_gemv_iq4_nl": (INT, [P, I64, P, P, P, P, P, I64, I64, I64, INT, P]),
    "b2q_gemv_q4_k": (INT, [P, I64, P, P, P, P, P, I64, I64, I64, INT, P]),
    "b2q_quant_gemv": (INT, [INT, P, I64, P, P, I64, P, P, P, I64, I64, I64, P]),
    "b2q_workspace_size": (ctypes.c_size_t, [INT, I64, I64, I64]),
    "b2q_pinned_workspace_size": (ctypes.c_size_t, [INT, I64, I64, I64]),
    "b2q_quant_gemv_pinned": (INT, [INT, P, I64, P, P, I64, P, I64, I64, I64, P, ctypes.c_size_t, P]),
    "b2q_host_device_pointer": (INT, [P, ctypes.POINTER(ctypes.c_void_p)]),
    "b2q_stage_pinned": (INT, [P, I64, P, I64, I64, P]),
    "b2q_split_blocks": (INT, [INT, P, I64, I64, P, I64, P, P]),
    "b2q_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "b2q_quant_gemv_splitk_noalloc": (INT, [INT, P, I64, P, P, I64, P, I64, I64, I64, INT, P]),
    "b2q_quant_gemv_ws": (INT, [INT, P, I64, P, P, I64, P, P, P, I64, I64, I64, P, ctypes.c_size_t, P]),
    "b2q_gemv_allgather": (INT, [INT, P, I64, P, P, I64, P, P, P, I64, P, P, I64, I64, I64, I64, I64, INT, INT,
                                 ctypes.c_longlong, P]),
    "b2q_set_tuning": (INT, [INT, INT, INT]),
    "b2q_set_pipeline": (INT, [INT, INT]),
    "b2q_set_warps": (INT, [INT]),
    "b2q_set_cluster": (INT, [INT]),
    "b2q_set_gemm_min_columns": (INT, [INT]),
    "b2q_set_gemm_schedule": (INT, [INT]),
    "b2q_set_splitk": (INT, [INT]),
    "b2q_device_error": (INT, [ctypes.POINTER(ctypes.c_int), INT]),
    "b2q_ipc_get_handle": (INT, [P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "b2q_ipc_open_handle": (INT, [P, ctypes.POINTER(ctypes.c_void_p)]),
    "b2q_ipc_close_handle": (INT, [P]),
    "b2q_probe_dp4a": (INT, [P, P, P, P, I64, P]),
    "b2q_decode_q4_0": (INT, [P, P, I64, P]),
    "b2q_decode_tq2_0": (INT, [P, P, I64, P]),
}


class B2QError(RuntimeError):
    """A C-ABI call returned a nonzero status; `.code` holds it."""

    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


_lib = None


def load():
    """The loaded library (raises FileNotFoundError with the build command if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `python -m comp_b200.build` (needs nvcc)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error():
    buf = ctypes.create_string_buffer(512)
    load().b2q_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def call(name, *args):
    """Calls a status-returning entry point; raises ValueError for argument errors, B2QError otherwise."""
    rc = getattr(load(), name)(*args)
    if rc != B2Q_OK:
        msg = last_error()
        if rc in (-1, -2, -4):
            raise ValueError(f"{name}: {msg}")
        raise B2QError(rc, msg)
    return rc


def launch_count():
    return int(load().b2q_launch_count())


def version():
    return load().b2q_version().decode()
