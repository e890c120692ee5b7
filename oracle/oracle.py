"""TEST INFRASTRUCTURE ONLY: Python front end of the ECF8 oracle.

Wraps oracle/liboracle.so (the C restatement of the reference decode kernel
dfloat/run/decode.cu:16-211 and packer dfloat/utils.py:373-499) and the
reference kernel compiled unmodified into oracle/_ref/libref_decode.so.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference arm may import this module; the product never does.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_decode.so")

_p = ctypes.c_void_p
_ll = ctypes.c_longlong
_lib = None
_ref = None


def build():
    """Builds liboracle.so (and _ref/ when the reference checkout exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        L.oracle_decode.restype = _ll
        L.oracle_decode.argtypes = [_p, ctypes.c_int, _p, _ll, _p, _p, _ll, _p, _ll, _p, _ll,
                                    ctypes.c_int, ctypes.c_int]
        L.oracle_encode_sizes.restype = ctypes.c_int
        L.oracle_encode_sizes.argtypes = [_p, _ll, _p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(_ll), ctypes.POINTER(_ll), ctypes.POINTER(_ll)]
        L.oracle_encode.restype = ctypes.c_int
        L.oracle_encode.argtypes = [_p, _ll, _p, _p, ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
                                    ctypes.c_int, _p, _p, _ll, _p]
        L.oracle_split.restype = None
        L.oracle_split.argtypes = [_p, _ll, _p, _p]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a.size else None


def decode(s, n_threads=0, out=None):
    """Decodes a stream dict (luts, encoded, packed, gaps, output_positions
    numpy arrays) on the CPU.  Returns (bytes u8[n], zero_length_events)."""
    luts = np.ascontiguousarray(s["luts"], np.uint8)
    enc = np.ascontiguousarray(s["encoded"], np.uint8)
    packed = np.ascontiguousarray(s["packed"], np.uint8)
    op = np.ascontiguousarray(s["output_positions"], np.uint64)
    gaps = np.ascontiguousarray(s["gaps"], np.uint8)
    n = packed.size * 2
    if out is None:
        out = np.zeros(n, np.uint8)
    tpb = int(s.get("threads_per_block", 512))
    z = lib().oracle_decode(_ptr(luts), luts.shape[0], _ptr(enc), enc.size, _ptr(packed), _ptr(op),
                            op.size, _ptr(gaps), gaps.size, _ptr(out), n, tpb, n_threads)
    if z < 0:
        raise ValueError("oracle_decode rejected the stream")
    return out, int(z)


def table_arrays(table_symbols, table_bits, table_values):
    bits = np.zeros(16, np.uint8)
    vals = np.zeros(16, np.uint32)
    for s, b, v in zip(table_symbols, table_bits, table_values):
        bits[int(s)] = b
        vals[int(s)] = v
    return bits, vals


def encode(exps, bits, vals, eof_bits, eof_val, bytes_per_thread=8, threads_per_block=512):
    """Packs exponents like dfloat/utils.py:373-499; returns (encoded, gaps, op)."""
    ex = np.ascontiguousarray(exps, np.uint8)
    bits = np.ascontiguousarray(bits, np.uint8)
    vals = np.ascontiguousarray(vals, np.uint32)
    nb, ng, nop = _ll(), _ll(), _ll()
    L = lib()
    if L.oracle_encode_sizes(_ptr(ex), ex.size, _ptr(bits), eof_bits, bytes_per_thread,
                             threads_per_block, ctypes.byref(nb), ctypes.byref(ng), ctypes.byref(nop)):
        raise ValueError("a symbol that occurs has no code")
    enc = np.zeros(nb.value, np.uint8)
    gaps = np.zeros(max(ng.value, 1), np.uint8)
    op = np.zeros(nop.value, np.uint64)
    L.oracle_encode(_ptr(ex), ex.size, _ptr(bits), _ptr(vals), eof_bits, eof_val, bytes_per_thread,
                    threads_per_block, _ptr(enc), _ptr(gaps), ng.value, _ptr(op))
    return enc, gaps[:ng.value], op


def split(fp8_u8):
    w = np.ascontiguousarray(fp8_u8, np.uint8)
    e = np.empty(w.size, np.uint8)
    p = np.empty(w.size // 2, np.uint8)
    lib().oracle_split(_ptr(w), w.size, _ptr(e), _ptr(p))
    return e, p


def reference_kernel_terminates(luts):
    """True when every 16-bit pattern resolves, through the LUTs, to a code of
    non-zero length -- the condition for the reference kernel
    (decode.cu:85-112) to terminate on arbitrary bits after the EOF code.
    Rows past n_luts read as 0 (the harness pads the LUT buffer)."""
    luts = np.asarray(luts, np.uint8)
    n = luts.shape[0]
    lens = luts[n - 1]
    padded = np.zeros((18, 256), np.uint8)
    padded[:n] = luts
    for b in range(256):
        d = int(luts[0, b])
        if d >= 240:
            row = padded[256 - d]
            if np.any(lens[row] == 0):
                return False
        elif lens[d] == 0:
            return False
    return True


def ref_lib():
    """ctypes handle of the reference kernel built from the reference sources."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB):
            raise FileNotFoundError(REF_LIB)
        L = ctypes.CDLL(REF_LIB)
        L.ref_decode_launch.restype = ctypes.c_int
        L.ref_decode_launch.argtypes = [_p, _p, _p, _p, _p, _p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, _p]
        _ref = L
    return _ref


def max_threads():
    return lib().oracle_max_threads()


def luts_from_table(table):
    """Restates dfloat/utils.py:270-370 (LUTs from a code table) in the same
    steps: prefixes "" plus the 8-bit leading strings of the longer codes in
    table order, one carry-forward row per prefix, then the length row."""
    items = [(s, b, v) for s, (b, v) in table.items() if isinstance(s, (int, np.integer))]
    prefixes = [""]
    for s, bits, val in items:
        binary = bin(val)[2:].rjust(bits, "0")
        plen = (bits - 1) - (bits - 1) % 8
        if binary[:plen] not in prefixes:
            prefixes.append(binary[:plen])
    prefixes.sort(key=len)
    luts = np.zeros((len(prefixes), 256), np.uint8)
    for pi, prefix in enumerate(prefixes):
        nb = len(prefix) // 8
        keys = {}
        for s, bits, val in items:
            binary = bin(val)[2:].rjust(bits, "0")
            if not binary.startswith(prefix):
                continue
            if (bits - 1) // 8 == nb:
                k, v = int(binary[nb * 8:].ljust(8, "0"), 2), s
            else:
                k, v = int(binary[nb * 8:nb * 8 + 8], 2), 256 - prefixes.index(binary[:nb * 8 + 8])
            if k in keys and keys[k] != v:
                raise ValueError("conflicting LUT keys")
            keys[k] = v
        cur = 0
        for b in range(256):
            cur = keys.get(b, cur)
            luts[pi, b] = cur
    lens = np.zeros((1, 256), np.uint8)
    for s, bits, _ in items:
        lens[0, s] = bits
    return np.concatenate([luts, lens], axis=0)
