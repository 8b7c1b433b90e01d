"""Zstandard oracle (TEST INFRASTRUCTURE ONLY, see ``oracle/__init__.py``).

The reference decodes zstd data with the `zstd` crate 0.13.3 (Cargo.lock),
which binds libzstd through zstd-sys 2.0.16+zstd.1.5.7: HoloTensorReader::
read_fragment (crates/haagenti-hct/src/holotensor.rs:2081-2091) and
GpuDecompressor::try_zstd_decompress (crates/haagenti-cuda/src/
decompress.rs:296-319) both call `zstd::decode_all`.  That library is the
decoder whose outputs the GPU path must reproduce; here it is the system
libzstd (1.5.x, loaded with ctypes), used to make test frames and to decode
them on the CPU.  The frame format it implements is RFC 8878.
"""
from __future__ import annotations

import ctypes as C

_lib = None

# ZSTD_cParameter values (zstd.h)
C_LEVEL = 100
C_WINDOW_LOG = 101
C_CONTENT_SIZE = 200
C_CHECKSUM = 201


def lib():
    global _lib
    if _lib is None:
        for name in ("libzstd.so.1", "libzstd.so"):
            try:
                _lib = C.CDLL(name)
                break
            except OSError:
                continue
        if _lib is None:
            raise OSError("libzstd not found")
        L = _lib
        L.ZSTD_compressBound.restype = C.c_size_t
        L.ZSTD_compressBound.argtypes = [C.c_size_t]
        L.ZSTD_isError.restype = C.c_uint
        L.ZSTD_isError.argtypes = [C.c_size_t]
        L.ZSTD_getErrorName.restype = C.c_char_p
        L.ZSTD_getErrorName.argtypes = [C.c_size_t]
        L.ZSTD_createCCtx.restype = C.c_void_p
        L.ZSTD_freeCCtx.argtypes = [C.c_void_p]
        L.ZSTD_CCtx_setParameter.restype = C.c_size_t
        L.ZSTD_CCtx_setParameter.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.ZSTD_compress2.restype = C.c_size_t
        L.ZSTD_compress2.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        L.ZSTD_decompress.restype = C.c_size_t
        L.ZSTD_decompress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        L.ZSTD_versionNumber.restype = C.c_uint
    return _lib


def version() -> int:
    return int(lib().ZSTD_versionNumber())


def compress(data: bytes, level: int = 3, checksum: bool = False, content_size: bool = True,
             window_log: int = 0) -> bytes:
    L = lib()
    data = bytes(data)
    cctx = L.ZSTD_createCCtx()
    try:
        for p, v in ((C_LEVEL, level), (C_CHECKSUM, int(checksum)),
                     (C_CONTENT_SIZE, int(content_size))):
            if L.ZSTD_isError(L.ZSTD_CCtx_setParameter(cctx, p, v)):
                raise ValueError(f"zstd parameter {p}={v}")
        if window_log and L.ZSTD_isError(L.ZSTD_CCtx_setParameter(cctx, C_WINDOW_LOG, window_log)):
            raise ValueError("zstd window log")
        cap = L.ZSTD_compressBound(len(data)) + 64
        out = C.create_string_buffer(cap)
        n = L.ZSTD_compress2(cctx, out, cap, data, len(data))
        if L.ZSTD_isError(n):
            raise ValueError(L.ZSTD_getErrorName(n).decode())
        return out.raw[:n]
    finally:
        L.ZSTD_freeCCtx(cctx)


def decompress(data: bytes, capacity: int):
    """(True, bytes) or (False, error name): ZSTD_decompress of every frame."""
    L = lib()
    data = bytes(data)
    out = C.create_string_buffer(max(capacity, 1))
    n = L.ZSTD_decompress(out, capacity, data, len(data))
    if L.ZSTD_isError(n):
        return False, L.ZSTD_getErrorName(n).decode()
    return True, out.raw[:n]


def decompress_into(data: bytes, buf) -> int:
    """ZSTD_decompress into a preallocated ctypes buffer: bytes written, or -1."""
    L = lib()
    n = L.ZSTD_decompress(buf, len(buf), data, len(data))
    return -1 if L.ZSTD_isError(n) else int(n)
