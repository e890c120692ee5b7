"""ctypes binding of the ECF8 CUDA library (C ABI in include/ecf8.h).

The library is the only implementation of the decode path: if it is missing
or fails to load, every entry point raises instead of falling back to
anything else.
"""

import ctypes
import os
import threading

from .build import LIB_NAME, PKG

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_TOO_LARGE = 4
NOALLOC_MAX_ELEMENTS = 268435456

ABI_VERSION = 8
TABLE_BYTES = 86544  # prepared decode table (ecf8_build_table)
MAX_LUTS = 18
MAX_BATCH = 256
DECODE_OVERLAP_PREVIOUS = 1  # ecf8_decode_batch_flags: may start while the stream's previous kernel runs
DECODE_CTAS_SHIFT = 16  # ecf8_decode_batch_flags bits 31..16: at most this many CTAs (0: one per SM)

THREADS_PER_BLOCK = 512
BYTES_PER_THREAD = 8


def decode_ctas(n):
    """ecf8_decode_batch_flags bits for a launch of at most n CTAs (1..65535)."""
    if not 1 <= n <= 0xFFFF:
        raise ValueError("the CTA limit is 1..65535")
    return n << DECODE_CTAS_SHIFT


_c_u8p = ctypes.c_void_p
_i64 = ctypes.c_int64


class Ecf8Stream(ctypes.Structure):
    """Mirror of `ecf8_stream` (include/ecf8.h)."""

    _fields_ = [
        ("luts", ctypes.c_void_p),
        ("n_luts", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("encoded", ctypes.c_void_p),
        ("n_bytes", ctypes.c_int64),
        ("packed_other_4bits", ctypes.c_void_p),
        ("output_positions", ctypes.c_void_p),
        ("n_output_positions", ctypes.c_int64),
        ("gaps", ctypes.c_void_p),
        ("n_gap_bytes", ctypes.c_int64),
        ("outputs", ctypes.c_void_p),
        ("n_elements", ctypes.c_int64),
        ("table", ctypes.c_void_p),
    ]


# Every symbol include/ecf8.h declares: name -> (restype, argtypes).
SIGNATURES = {
    "ecf8_decode": (ctypes.c_int, [_c_u8p, _c_u8p, _c_u8p, _c_u8p, _c_u8p, _c_u8p, ctypes.c_int,
                                   _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ecf8_build_table": (ctypes.c_int, [_c_u8p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "ecf8_decode_batch": (ctypes.c_int, [ctypes.POINTER(Ecf8Stream), ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_void_p]),
    "ecf8_decode_batch_flags": (ctypes.c_int, [ctypes.POINTER(Ecf8Stream), ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p]),
    "ecf8_encode_workspace_bytes": (ctypes.c_int64, [_i64]),
    "ecf8_encode_plan": (ctypes.c_int, [_c_u8p, _i64, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p]),
    "ecf8_encode_emit": (ctypes.c_int, [_c_u8p, _i64, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                                        ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p, _c_u8p, _i64, _i64,
                                        _c_u8p, _i64, ctypes.c_void_p, _i64, ctypes.c_void_p]),
    "ecf8_encode_noalloc": (ctypes.c_int, [_c_u8p, _i64, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                                           ctypes.c_int, ctypes.c_uint32, _c_u8p, _i64, _c_u8p, _i64,
                                           ctypes.c_void_p, _i64, ctypes.c_void_p, ctypes.c_void_p]),
    "ecf8_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ecf8_last_cuda_error": (ctypes.c_int, []),
    "ecf8_abi_version": (ctypes.c_int, []),
}

_lock = threading.Lock()
_lib = None


def library_path():
    return os.path.join(PKG, LIB_NAME)


def lib():
    """The loaded library; raises RuntimeError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"ECF8 CUDA library {path} is missing; build it with "
                    "`python -m ecf8_b200.build` (the decode path has no fallback)")
            handle = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            if handle.ecf8_abi_version() != ABI_VERSION:
                raise RuntimeError("ECF8 CUDA library ABI version mismatch")
            _lib = handle
    return _lib


class Ecf8Error(RuntimeError):
    def __init__(self, status, what):
        L = lib()
        msg = L.ecf8_status_string(status).decode()
        if status == ERR_CUDA:
            msg += f" (cudaError {L.ecf8_last_cuda_error()})"
        super().__init__(f"{what}: {msg}")
        self.status = status


def check(status, what):
    if status != OK:
        raise Ecf8Error(status, what)
