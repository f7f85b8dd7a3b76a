"""ctypes binding of the C ABI in include/m3ssd.h (libm3ssd.so, built in-tree for sm_100a).

This is the same binding a maintainer of the reference would add: plain structs of pointers,
int64 sizes and strides, and an int status that becomes a Python exception.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libm3ssd.so")

M3SSD_X_COMPLEX = 0x1
M3SSD_PREC_AUTO = 0x0
M3SSD_PREC_FP32 = 0x10
M3SSD_PREC_TENSOR = 0x20
M3SSD_Y_BF16 = 0x100

STATUS_NAMES = {
    0: "OK", 1: "ERR_NULL", 2: "ERR_SHAPE", 3: "ERR_CHUNK", 4: "ERR_DIM_LIMIT", 5: "ERR_ALIGN",
    6: "ERR_WORKSPACE", 7: "ERR_LAUNCH", 8: "ERR_DEVICE", 9: "ERR_FLAGS", 10: "ERR_OVERFLOW",
    11: "ERR_SCRATCH_LIMIT",
}

I64x3 = ctypes.c_int64 * 3
I64x4 = ctypes.c_int64 * 4


class Problem(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("seqlen", ctypes.c_int64),
                ("nheads", ctypes.c_int64), ("headdim", ctypes.c_int64),
                ("dstate", ctypes.c_int64), ("chunk", ctypes.c_int64),
                ("flags", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class FwdArgs(ctypes.Structure):
    _fields_ = [("prob", Problem),
                ("x", ctypes.c_void_p), ("x_strides", I64x4),
                ("A", ctypes.c_void_p),
                ("B", ctypes.c_void_p), ("b_strides", I64x4),
                ("C", ctypes.c_void_p), ("c_strides", I64x4),
                ("dt", ctypes.c_void_p), ("dt_strides", I64x3),
                ("y", ctypes.c_void_p),
                ("states", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("prob", Problem),
                ("x", ctypes.c_void_p), ("x_strides", I64x4),
                ("A", ctypes.c_void_p),
                ("B", ctypes.c_void_p), ("b_strides", I64x4),
                ("C", ctypes.c_void_p), ("c_strides", I64x4),
                ("dt", ctypes.c_void_p), ("dt_strides", I64x3),
                ("dy", ctypes.c_void_p), ("dy_strides", I64x4),
                ("states", ctypes.c_void_p),
                ("dx", ctypes.c_void_p), ("dA", ctypes.c_void_p),
                ("dB", ctypes.c_void_p), ("dC", ctypes.c_void_p), ("ddt", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


I64x2 = ctypes.c_int64 * 2


class ProjFwdArgs(ctypes.Structure):
    _fields_ = [("prob", Problem),
                ("proj", ctypes.c_void_p), ("proj_strides", I64x2),
                ("A", ctypes.c_void_p),
                ("y", ctypes.c_void_p),
                ("states", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


class ProjBwdArgs(ctypes.Structure):
    _fields_ = [("prob", Problem),
                ("proj", ctypes.c_void_p), ("proj_strides", I64x2),
                ("A", ctypes.c_void_p),
                ("dy", ctypes.c_void_p), ("dy_strides", I64x4),
                ("states", ctypes.c_void_p),
                ("dproj", ctypes.c_void_p), ("dproj_strides", I64x2),
                ("dA", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


# every symbol include/m3ssd.h declares, with its ctypes signature
SIGNATURES = {
    "m3ssd_abi_version": (ctypes.c_int, []),
    "m3ssd_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "m3ssd_check_problem": (ctypes.c_int, [ctypes.POINTER(Problem)]),
    "m3ssd_states_bytes": (ctypes.c_size_t, [ctypes.POINTER(Problem)]),
    "m3ssd_fwd_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Problem)]),
    "m3ssd_bwd_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Problem)]),
    "m3ssd_fwd": (ctypes.c_int, [ctypes.POINTER(FwdArgs), ctypes.c_void_p]),
    "m3ssd_bwd": (ctypes.c_int, [ctypes.POINTER(BwdArgs), ctypes.c_void_p]),
    "m3ssd_fwd_path": (ctypes.c_char_p, [ctypes.POINTER(Problem)]),
    "m3ssd_bwd_path": (ctypes.c_char_p, [ctypes.POINTER(Problem)]),
    "m3ssd_launch_count": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.c_int]),
    "m3ssd_fwd_static_scratch": (ctypes.c_int, [ctypes.POINTER(FwdArgs), ctypes.c_void_p]),
    "m3ssd_fwd_proj": (ctypes.c_int, [ctypes.POINTER(ProjFwdArgs), ctypes.c_void_p]),
    "m3ssd_bwd_proj": (ctypes.c_int, [ctypes.POINTER(ProjBwdArgs), ctypes.c_void_p]),
    "m3ssd_fwd_state": (ctypes.c_int, [ctypes.POINTER(FwdArgs), ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p]),
    "m3ssd_bwd_state": (ctypes.c_int, [ctypes.POINTER(BwdArgs), ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p]),
    "m3ssd_selftest_bounded_waits": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t,
                                                    ctypes.c_void_p]),
}

_lib = None


def load(path: str | None = None):
    """Load libm3ssd.so (once) and bind its signatures. Raises if the library is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(
            f"m3ssd CUDA library not found at {p}; build it with "
            "`python mamba-3-lite_b200/m3ssd/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.m3ssd_abi_version() != 1:
        raise RuntimeError("m3ssd ABI version mismatch")
    if path is None:
        _lib = lib
    return lib


class M3SsdError(RuntimeError):
    def __init__(self, status: int, lib=None):
        lib = lib or load()
        msg = lib.m3ssd_strerror(int(status)).decode()
        super().__init__(f"{msg} (status {status}: {STATUS_NAMES.get(status, '?')})")
        self.status = status


def check(status: int):
    if status != 0:
        raise M3SsdError(status)
