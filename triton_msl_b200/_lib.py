"""ctypes binding of libb2msl.so (the C ABI declared in include/b2msl.h).

This is the FFI layer a Python caller of the reference's hot path binds: plain
pointers, sizes and a CUDA stream handle. Every call is checked; a non-zero
status raises with the library's own message (the reference raises
MetalNonRecoverableError instead of returning wrong numbers,
triton_msl/errors.py:82-102). There is no fallback: if the library is missing
or cannot load, calls raise.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("B2MSL_LIBRARY", PKG / "libb2msl.so"))

B2_OK, B2_EINVAL, B2_EUNSUPPORTED, B2_ELAUNCH, B2_ETIMEOUT = 0, -1, -2, -3, -4
B2_F32, B2_F16, B2_BF16, B2_I64 = 0, 1, 2, 3
STATUS_TIMEOUT_TMA, STATUS_TIMEOUT_MMA, STATUS_TIMEOUT_EPI, STATUS_TIMEOUT_SLOT = 1, 2, 4, 8
ACT = {"none": 0, "relu": 1, "gelu": 2, "gelu_tanh": 3, "silu": 4, "softmax": 5}
# b2_gemm_epilogue op codes (B2_EPI_* in include/b2msl.h) and their constant counts
EPI = {"add": (1, 1), "sub": (2, 1), "rsub": (3, 1), "mul": (4, 1), "div": (5, 1),
       "rdiv": (6, 1), "add_bias": (7, 0), "mul_bias": (8, 0), "max": (9, 1), "min": (10, 1),
       "maxnum": (11, 1), "minnum": (12, 1), "clamp": (13, 2), "clampnum": (14, 2),
       "neg": (15, 0), "exp": (16, 0), "exp2": (17, 0), "log": (18, 0), "log2": (19, 0),
       "sqrt": (20, 0), "rsqrt": (21, 0), "sin": (22, 0), "cos": (23, 0), "erf": (24, 0),
       "tanh": (25, 0), "floor": (26, 0), "ceil": (27, 0), "abs": (28, 0), "relu": (29, 0),
       "gelu": (30, 0), "gelu_tanh": (31, 0), "silu": (32, 0), "sigmoid": (33, 0),
       "fma": (34, 2)}
EPI_MAX_OPS = 16
ROW_OPS = {"softmax": 0, "layernorm": 1, "rmsnorm": 2, "sum": 3, "max": 4,
           "argmax": 5, "min": 6, "argmin": 7}

# Every symbol include/b2msl.h declares, with its ctypes signature.
_c_i64p = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "b2_version": (ctypes.c_char_p, []),
    "b2_last_error": (ctypes.c_char_p, []),
    "b2_last_kernel": (ctypes.c_char_p, []),
    "b2_fa_fwd": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 4
                  + [_c_i64p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "b2_gemm": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
                + [_c_i64p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "b2_gemm_epilogue": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
                         + [_c_i64p, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float),
                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "b2_reduce_axis": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
                       + [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                                  ctypes.c_void_p]),
    "b2_row_op": (ctypes.c_int, [ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 4
                  + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                     ctypes.c_void_p]),
    "b2_row_reduce_noalloc": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
                              + [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_void_p]),
    "b2_test_stalled_gemm": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3
                             + [ctypes.c_uint64, ctypes.c_void_p]),
    "b2_query_workspace": (ctypes.c_size_t, [ctypes.c_int] + [ctypes.c_int64] * 4),
    "b2_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_uint32)]),
}

_lock = threading.Lock()
_lib = None


class B2Error(RuntimeError):
    """A b2msl entry point returned a failure status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed (status {status}): {msg}")
        self.status = status


class B2Unsupported(B2Error, NotImplementedError):
    """The request is valid but not implemented (B2_EUNSUPPORTED)."""


def lib() -> ctypes.CDLL:
    """Load (building in-tree first if absent and nvcc exists) and return the library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists() and os.environ.get("B2MSL_NO_AUTOBUILD") != "1":
                from . import _build
                _build.build()
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with "
                                   "`python -m triton_msl_b200._build`")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status == B2_OK:
        return
    msg = lib().b2_last_error().decode()
    if status == B2_EUNSUPPORTED:
        raise B2Unsupported(fn, status, msg)
    raise B2Error(fn, status, msg)


def i64_array(vals) -> ctypes.Array:
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * len(vals))(*vals)


def last_kernel() -> str:
    return lib().b2_last_kernel().decode()


def device_status(device: int, clear: bool = True) -> int:
    out = ctypes.c_uint32(0)
    st = lib().b2_device_status(int(device), 1 if clear else 0, ctypes.byref(out))
    if st not in (B2_OK, B2_ETIMEOUT):
        check("b2_device_status", st)
    return int(out.value)
