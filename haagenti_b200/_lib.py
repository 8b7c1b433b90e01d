"""ctypes binding of libhct_b200.so (include/hct_b200.h).

The shared library is the product; this module only declares its C ABI.
It fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhct_b200.so")

OK = 0
UNEXPECTED_EOF = 1
BUFFER_TOO_SMALL = 2
ZERO_OFFSET = 3
OFFSET_BEYOND = 4
INVALID_ARGUMENT = 16
CORRUPTED = 17
CHECKSUM = 18
UNSUPPORTED = 19
CUDA = 20
NO_DEVICE = 21
TIMEOUT = 22
OUT_OF_MEMORY = 23
SIZE_MISMATCH = 24

F32, F16, BF16 = 0, 1, 2
FLAG_SPECTRAL_Q4 = 0x0100


class Lz4Block(C.Structure):
    _fields_ = [("src_off", C.c_uint64), ("dst_off", C.c_uint64), ("src_len", C.c_uint32),
                ("dst_cap", C.c_uint32), ("out_size", C.c_uint32), ("reserved", C.c_uint32)]


class BlockStatus(C.Structure):
    _fields_ = [("code", C.c_int32), ("reserved", C.c_int32), ("position", C.c_uint64),
                ("provided", C.c_uint64), ("written", C.c_uint64)]


class Error(C.Structure):
    _fields_ = [("code", C.c_int32), ("block", C.c_int32), ("position", C.c_uint64),
                ("required", C.c_uint64), ("provided", C.c_uint64), ("message", C.c_char * 192)]


class Header(C.Structure):
    _fields_ = [("version", C.c_uint32), ("algorithm", C.c_uint8), ("dtype", C.c_uint8),
                ("flags", C.c_uint16), ("original_size", C.c_uint64),
                ("compressed_size", C.c_uint64), ("block_size", C.c_uint32),
                ("num_blocks", C.c_uint32), ("rank", C.c_uint32), ("reserved", C.c_uint32),
                ("shape", C.c_uint64 * 4), ("quant_meta", C.c_uint8 * 8),
                ("has_quant_meta", C.c_uint32), ("reserved2", C.c_uint32)]


class HoloInfo(C.Structure):
    _fields_ = [("encoding", C.c_uint8), ("compression", C.c_uint8), ("flags", C.c_uint16),
                ("total_fragments", C.c_uint16), ("min_fragments", C.c_uint16),
                ("original_size", C.c_uint64), ("seed", C.c_uint64), ("dtype", C.c_uint8),
                ("ndim", C.c_uint8), ("inline_format", C.c_uint16), ("reserved", C.c_uint32),
                ("shape", C.c_uint64 * 7), ("quality_curve", C.c_float * 4),
                ("rows", C.c_uint64), ("cols", C.c_uint64)]


class Int4Job(C.Structure):
    _fields_ = [("d_data", C.c_void_p), ("data_len", C.c_uint64), ("num_elements", C.c_uint64),
                ("d_out", C.c_void_p)]


class KernelStats(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_uint64), ("total_ms", C.c_double),
                ("work", C.c_double)]


# Every exported symbol with (restype, argtypes); tests check the list
# against include/hct_b200.h.
_vp, _sz, _u8p = C.c_void_p, C.c_size_t, C.c_void_p
SIGNATURES = {
    "hct_b200_abi_version": (C.c_int, []),
    "hct_b200_status_string": (C.c_char_p, [C.c_int]),
    "hct_b200_ctx_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "hct_b200_ctx_destroy": (None, [_vp]),
    "hct_b200_ctx_reserve": (C.c_int, [_vp, C.c_uint64, C.c_uint64]),
    "hct_b200_ctx_set_idct": (C.c_int, [_vp, C.c_int]),
    "hct_b200_ctx_profile": (C.c_int, [_vp, C.c_int]),
    "hct_b200_ctx_profile_read": (C.c_int, [_vp, C.POINTER(KernelStats), C.c_int,
                                            C.POINTER(C.c_int)]),
    "hct_b200_lz4_max_compressed_size": (C.c_size_t, [C.c_size_t]),
    "hct_b200_lz4_compress_block": (C.c_int, [_u8p, _sz, _u8p, _sz, C.POINTER(C.c_size_t)]),
    "hct_b200_lz4_compress_chunks": (C.c_int, [_u8p, _sz, _sz, _u8p, _sz,
                                               C.POINTER(C.c_uint32)]),
    "hct_b200_quantize_int4": (C.c_int, [_vp, _sz, _u8p]),
    "hct_b200_quantize_int4_mp": (C.c_int, [_vp, _sz, _u8p]),
    "hct_b200_spectral_select": (C.c_int, [_vp, _sz, _sz, _u8p, _vp, C.POINTER(C.c_size_t)]),
    "hct_b200_lz4_decompress_blocks": (C.c_int, [_vp, _vp, C.c_uint32, _vp, _vp, C.c_uint64,
                                                 _vp]),
    "hct_b200_lz4_decompress_with_size": (C.c_int, [_vp, _u8p, _sz, _sz, _u8p,
                                                    C.POINTER(C.c_size_t), C.POINTER(Error)]),
    "hct_b200_lz4_decompress_to": (C.c_int, [_vp, _u8p, _sz, _u8p, _sz,
                                             C.POINTER(C.c_size_t), C.POINTER(Error)]),
    "hct_b200_dequantize_int4": (C.c_int, [_vp, _sz, _sz, _vp, C.c_int,
                                           C.POINTER(C.c_size_t), _vp]),
    "hct_b200_dequantize_int4_mp": (C.c_int, [_vp, _sz, _sz, _vp, C.c_int,
                                              C.POINTER(C.c_size_t), _vp]),
    "hct_b200_dequantize_int4_batch": (C.c_int, [C.POINTER(Int4Job), C.c_uint32, C.c_int,
                                                 C.POINTER(C.c_size_t), _vp]),
    "hct_b200_idct_2d": (C.c_int, [_vp, _vp, _vp, C.c_int, _sz, _sz, _vp]),
    "hct_b200_spectral_q4_decode": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _vp, C.c_int, _vp]),
    "hct_b200_spectral_q4_decode_noalloc": (C.c_int, [_vp, _sz, _sz, _sz, _vp, C.c_int, _vp]),
    "hct_b200_v3_open": (C.c_int, [_vp, _u8p, _sz, C.c_uint64, C.c_uint64,
                                   C.POINTER(C.c_void_p), C.POINTER(Error)]),
    "hct_b200_v3_num_fragments": (C.c_int, [_vp]),
    "hct_b200_v3_decode": (C.c_int, [_vp, _vp, C.c_int, _vp, C.POINTER(Error)]),
    "hct_b200_v3_close": (None, [_vp]),
    "hct_b200_hct_v3_decode": (C.c_int, [_vp, _u8p, _sz, C.c_uint64, C.c_uint64, _vp, C.c_int,
                                         _vp, C.POINTER(Error)]),
    "hct_b200_zstd_decompress_jobs": (C.c_int, [_vp, _vp, _vp, C.c_uint32, _vp, _vp, _vp]),
    "hct_b200_zstd_decompress": (C.c_int, [_vp, _u8p, _sz, _u8p, _sz, C.POINTER(C.c_size_t),
                                           C.POINTER(Error)]),
    "hct_b200_zstd_content_size": (C.c_int, [_u8p, _sz, C.POINTER(C.c_uint64)]),
    "hct_b200_holo_open": (C.c_int, [_vp, _u8p, _sz, C.POINTER(C.c_void_p), C.POINTER(Error)]),
    "hct_b200_holo_header": (C.c_int, [_vp, C.POINTER(HoloInfo)]),
    "hct_b200_holo_total_fragments": (C.c_int, [_vp]),
    "hct_b200_holo_predict_quality": (C.c_float, [_vp, C.c_uint32]),
    "hct_b200_holo_fragments_for_quality": (C.c_uint32, [_vp, C.c_float]),
    "hct_b200_holo_decode": (C.c_int, [_vp, C.c_uint32, _vp, C.c_int, _vp,
                                       C.POINTER(C.c_float), C.POINTER(Error)]),
    "hct_b200_holo_close": (None, [_vp]),
    "hct_b200_reader_open": (C.c_int, [_vp, _u8p, _sz, C.c_int, C.POINTER(C.c_void_p),
                                       C.POINTER(Error)]),
    "hct_b200_reader_upload": (C.c_int, [_vp, _u8p, _sz, _vp]),
    "hct_b200_reader_header": (C.c_int, [_vp, C.POINTER(Header)]),
    "hct_b200_reader_num_blocks": (C.c_uint32, [_vp]),
    "hct_b200_reader_decompress_all": (C.c_int, [_vp, _vp, _sz, C.POINTER(C.c_size_t), _vp,
                                                 C.POINTER(Error)]),
    "hct_b200_reader_decode": (C.c_int, [_vp, _vp, C.c_int, _vp, C.POINTER(Error)]),
    "hct_b200_reader_decode_async": (C.c_int, [_vp, _vp, C.c_int, _vp, C.POINTER(Error)]),
    "hct_b200_reader_wait": (C.c_int, [_vp, C.POINTER(Error)]),
    "hct_b200_reader_close": (None, [_vp]),
}

_lib = None


def load() -> C.CDLL:
    """Load libhct_b200.so; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m haagenti_b200.build` "
            "(the CUDA library is required; there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
