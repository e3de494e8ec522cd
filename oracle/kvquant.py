"""ORACLE — test infrastructure only.

ctypes wrapper of kvquant_oracle.c, the plain-C restatement of the
reference's INT8 KV compressor (KVCompressor::compress / decompress,
cascade_Code/cpp/src/cascade_core.cpp:908-967). The checker of the store's
INT8 tier-move kernels; the product never imports it.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .store_oracle import _load

_ready = False


def _lib():
    global _ready
    lib = _load()
    if not _ready:
        lib.kvq_compress.restype = C.c_uint64
        lib.kvq_compress.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        lib.kvq_decompress.restype = C.c_int
        lib.kvq_decompress.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p]
        lib.kvq_params.restype = None
        lib.kvq_params.argtypes = [C.c_int32, C.c_int32, C.POINTER(C.c_float), C.POINTER(C.c_int8)]
        _ready = True
    return lib


def compressed_size(size: int) -> int:
    """KVCompressor::compressed_size (include/cascade.hpp:410-412)."""
    return 8 + size // 2


def compress(data) -> bytes:
    """[f32 scale][i8 zero_point][3 zero bytes][size/2 x i8]; size >= 2."""
    a = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray))
                             else np.asarray(data, np.uint8).reshape(-1))
    if a.size < 2:
        raise ValueError("compress needs at least one 16-bit value")
    out = np.zeros(compressed_size(a.size), np.uint8)
    _lib().kvq_compress(a.ctypes.data, a.size, out.ctypes.data)
    return out.tobytes()


def decompress(comp, orig_size: int) -> bytes | None:
    """(orig_size/2)*2 bytes, or None when comp is too short (the reference's
    `return false`)."""
    c = np.ascontiguousarray(np.frombuffer(bytes(comp), np.uint8))
    out = np.zeros(orig_size // 2 * 2, np.uint8)
    ok = _lib().kvq_decompress(c.ctypes.data if c.size else 0, c.size, orig_size, out.ctypes.data)
    return out.tobytes() if ok else None


def roundtrip(data) -> bytes:
    """What a get returns for a block that went through the INT8 DRAM tier."""
    b = bytes(np.asarray(data, np.uint8).reshape(-1)) if not isinstance(data, (bytes, bytearray)) else bytes(data)
    return decompress(compress(b), len(b))


def params(mn: int, mx: int) -> tuple[float, int]:
    s, z = C.c_float(), C.c_int8()
    _lib().kvq_params(mn, mx, C.byref(s), C.byref(z))
    return s.value, z.value
