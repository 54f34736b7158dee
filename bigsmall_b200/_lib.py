"""ctypes binding of libbsgpu.so, the sm_100a decode/encode engine.

The shared library is built in-tree (``bigsmall_b200/libbsgpu.so``) by
``bigsmall_b200.build.build()``.  There is no fallback: if the library or a
CUDA device is missing, every entry point raises.  The C declarations live in
``include/bsgpu.h``.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .exceptions import BsCorruptError, BsGpuError

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbsgpu.so")

BS_OK = 0
BS_E_INVALID_ARG = 1
BS_E_BAD_MAGIC = 2
BS_E_COUNT_MISMATCH = 3
BS_E_TRUNCATED = 4
BS_E_CORRUPT = 5
BS_E_CUDA = 6
BS_E_UNSUPPORTED = 7
BS_E_NOMEM = 8
BS_E_PRECISION = 9

DEV_BITS = {0x01: "header", 0x02: "freq", 0x04: "chunk_table", 0x08: "stream",
            0x10: "final_state", 0x20: "count"}

CODER_RANS = 0
CODER_TANS = 1
CODER_RANS_PAIR = 2
SE_SINGLE_KERNEL = 1
SE_TANS = 2
SE_PARALLEL = 3   # bf16_parallel_v1 blobs in a serial-format batch


class XcTensor(ctypes.Structure):
    """Mirror of ``bs_xc_tensor`` in include/bsgpu.h."""
    _fields_ = [
        ("d_blob", ctypes.c_void_p),
        ("blob_bytes", ctypes.c_uint64),
        ("d_out", ctypes.c_void_p),
        ("n_elems", ctypes.c_uint64),
        ("chunk_elems", ctypes.c_uint32),
        ("chunk_begin", ctypes.c_uint32),
        ("chunk_count", ctypes.c_uint32),
        ("coder_mask", ctypes.c_uint32),
        ("groups", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
    ]


class SeBlob(ctypes.Structure):
    """Mirror of ``bs_se_blob`` in include/bsgpu.h."""
    _fields_ = [
        ("codec", ctypes.c_int),
        ("h_blob", ctypes.c_void_p),
        ("blob_bytes", ctypes.c_uint64),
        ("n_weights", ctypes.c_uint64),
        ("d_blob", ctypes.c_void_p),
        ("d_out", ctypes.c_void_p),
    ]


# every symbol include/bsgpu.h declares, with its ctypes signature
_P, _U64, _I, _U32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32
SIGNATURES = {
    "bs_version": (_I, []),
    "bs_last_error": (ctypes.c_char_p, []),
    "bs_status_string": (ctypes.c_char_p, [_I]),
    "bs_xc_plan_create": (_I, [ctypes.POINTER(XcTensor), _I, _I, ctypes.POINTER(_P)]),
    "bs_plan_decode": (_I, [_P, _P]),
    "bs_plan_decode_timed": (_I, [_P, _P, _P, _P]),
    "bs_plan_decode_after": (_I, [_P, _P, _P, _P]),
    "bs_plan_decode_handoff": (_I, [_P, _P, _P, _P, _P, _P]),
    "bs_plan_check": (_I, [_P, _P, ctypes.POINTER(_U32)]),
    "bs_plan_n_tensors": (_I, [_P]),
    "bs_plan_launch_count": (_I, [_P, ctypes.POINTER(_U64)]),
    "bs_plan_set_max_ctas": (_I, [_P, _I]),
    "bs_plan_destroy": (_I, [_P]),
    "bs_xc_decode_noalloc": (_I, [ctypes.POINTER(XcTensor), _I, _P, ctypes.POINTER(_U32)]),
    "bs_par_plan_create": (_I, [_P, _U64, _U64, _P, _P, _I, ctypes.POINTER(_P)]),
    "bs_xc_encode_bound": (_I, [_U64, _U32, _U32, ctypes.POINTER(_U64)]),
    "bs_xc_encode_workspace": (_I, [_U64, _U32, _U32, _I, ctypes.POINTER(_U64)]),
    "bs_xc_encode": (_I, [_P, _U64, _I, _I, _U32, _U32, _P, _U64, _P, _P, _U64, _P]),
    "bs_se_plan_create": (_I, [_I, _P, _U64, _U64, _P, _P, _I, ctypes.POINTER(_P)]),
    "bs_se_parse": (_I, [_I, _P, _U64, _U64, ctypes.POINTER(_U32)]),
    "bs_se_plan_create_many": (_I, [ctypes.POINTER(SeBlob), _I, _I, ctypes.POINTER(_P)]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load libbsgpu.so (once).  Raises ImportError if it is not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise ImportError(
                f"libbsgpu.so not found at {path}; build it with "
                "`python -c 'import bigsmall_b200.build as b; b.build()'` (nvcc, sm_100a)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().bs_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(status: int, what: str, device_status=None) -> None:
    """Raise the Python exception matching a C-ABI status."""
    if status == BS_OK:
        return
    msg = f"{what}: {last_error() or load().bs_status_string(status).decode()}"
    if status in (BS_E_BAD_MAGIC, BS_E_COUNT_MISMATCH, BS_E_TRUNCATED, BS_E_CORRUPT, BS_E_PRECISION):
        raise BsCorruptError(status, msg, device_status)
    if status == BS_E_INVALID_ARG:
        raise ValueError(msg)
    raise BsGpuError(status, msg, device_status)


def describe_device_status(word: int) -> str:
    return "|".join(name for bit, name in DEV_BITS.items() if word & bit) or "ok"
