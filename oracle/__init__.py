"""CPU parity oracle for the HCT weight-decode path.

TEST INFRASTRUCTURE ONLY: ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import this package; the product path
(``haagenti_b200``) never does.

It wraps ``liboracle.so`` (a C restatement of the reference's own Rust code,
see ``hct_oracle.c`` for the per-function citations) and adds, in Python:

* the HCT container writer/reader (crates/haagenti-hct/src/tensor.rs:275-1021),
* the composite "HCT-Q4" spectral payload encoder/decoder defined by this
  project from the reference's primitives (DCT -> top-k bitmap -> INT4 ->
  LZ4-wrapped HCT), and
* seeded generators for the benchmark configurations.

Parity of the IDCT against the reference is pinned to an f64 truth
(``scipy.fft.idctn(type=2, norm='ortho')``) and to the reference's C decoder
(``ref/c/hct_decoder.h``, compiled into ``oracle/_ref``) because the
reference's f32 rounding comes from rustfft 6.4.1, which is not available.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

OK, UNEXPECTED_EOF, BUFFER_TOO_SMALL, ZERO_OFFSET, OFFSET_BEYOND = 0, 1, 2, 3, 4
Q4_BLOCK_SIZE = 32
DEFAULT_BLOCK_SIZE = 16 * 1024  # tensor.rs:74


def reference_root() -> str | None:
    """The haagenti checkout the golden vectors and oracle/_ref come from:
    $HAAGENTI_REFERENCE, else a ``reference`` directory beside this
    repository; None when neither exists (as on a GPU box)."""
    cands = [os.environ.get("HAAGENTI_REFERENCE"),
             os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "ref", "c")):
            return os.path.abspath(c)
    return None


def build() -> str:
    """Compile liboracle.so (and the reference C decoder when its checkout is present)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    ref = reference_root()
    if ref:
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF_DIR={ref}/ref/c"], check=True)
    return _LIB_PATH


def _load() -> C.CDLL:
    if not os.path.exists(_LIB_PATH):
        build()
    lib = C.CDLL(_LIB_PATH)
    u8p = C.POINTER(C.c_uint8)
    f32p = C.POINTER(C.c_float)
    sz = C.c_size_t
    szp = C.POINTER(C.c_size_t)
    lib.orc_lz4_max_compressed_size.restype = sz
    lib.orc_lz4_max_compressed_size.argtypes = [sz]
    lib.orc_lz4_compress_block.restype = C.c_int
    lib.orc_lz4_compress_block.argtypes = [u8p, sz, u8p, sz, szp, szp]
    lib.orc_lz4_decompress_block.restype = C.c_int
    lib.orc_lz4_decompress_block.argtypes = [u8p, sz, u8p, sz, sz, szp, szp, szp]
    lib.orc_lz4_decompress_batch.restype = None
    lib.orc_lz4_decompress_batch.argtypes = [u8p, C.c_void_p, sz, u8p, C.c_void_p, C.c_int]
    lib.orc_lz4_compress_chunks.restype = C.c_int
    lib.orc_lz4_compress_chunks.argtypes = [u8p, sz, sz, u8p, sz, C.POINTER(C.c_uint32), C.c_int]
    lib.orc_f32_to_f16_bits.restype = C.c_uint16
    lib.orc_f32_to_f16_bits.argtypes = [C.c_float]
    lib.orc_f16_bits_to_f32.restype = C.c_float
    lib.orc_f16_bits_to_f32.argtypes = [C.c_uint16]
    lib.orc_int4_compressed_size.restype = sz
    lib.orc_int4_compressed_size.argtypes = [sz]
    lib.orc_quantize_int4.restype = None
    lib.orc_quantize_int4.argtypes = [f32p, sz, u8p]
    lib.orc_dequantize_int4.restype = sz
    lib.orc_dequantize_int4.argtypes = [u8p, sz, sz, f32p]
    lib.orc_dequantize_int4_threads.restype = sz
    lib.orc_dequantize_int4_threads.argtypes = [u8p, sz, sz, f32p, C.c_int]
    lib.orc_f32_to_f16_rne.restype = C.c_uint16
    lib.orc_f32_to_f16_rne.argtypes = [C.c_float]
    lib.orc_quantize_int4_mp.restype = None
    lib.orc_quantize_int4_mp.argtypes = [f32p, sz, u8p]
    lib.orc_dequantize_int4_mp.restype = sz
    lib.orc_dequantize_int4_mp.argtypes = [u8p, sz, sz, f32p]
    for name in ("orc_dct_1d", "orc_idct_1d"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = [f32p, f32p, sz]
    for name in ("orc_dct_2d", "orc_idct_2d"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = [f32p, f32p, sz, sz, C.c_int]
    lib.orc_retain_count.restype = sz
    lib.orc_retain_count.argtypes = [sz, C.c_float]
    lib.orc_topk_bitmap.restype = sz
    lib.orc_topk_bitmap.argtypes = [f32p, sz, sz, u8p, C.c_int]
    lib.orc_gather_retained.restype = sz
    lib.orc_gather_retained.argtypes = [f32p, sz, u8p, f32p]
    lib.orc_scatter_retained.restype = sz
    lib.orc_scatter_retained.argtypes = [f32p, sz, u8p, sz, f32p]
    lib.orc_popcount_bytes.restype = sz
    lib.orc_popcount_bytes.argtypes = [u8p, sz]
    lib.orc_num_threads.restype = C.c_int
    return lib


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _u8(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def _f32(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _as_u8(data) -> np.ndarray:
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    return np.frombuffer(bytes(data), dtype=np.uint8)


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---------------------------------------------------------------- LZ4 (block.rs)

def max_compressed_size(n: int) -> int:
    return int(lib().orc_lz4_max_compressed_size(n))


def lz4_compress_block(data) -> bytes:
    """block.rs:73 compress_block into a max_compressed_size buffer (compress.rs:60-76)."""
    src = _as_u8(data)
    cap = max_compressed_size(src.size)
    out = np.zeros(max(cap, 1), dtype=np.uint8)
    ol, req = C.c_size_t(0), C.c_size_t(0)
    rc = lib().orc_lz4_compress_block(_u8(src), src.size, _u8(out), cap, C.byref(ol), C.byref(req))
    if rc != OK:
        raise RuntimeError(f"compress_block failed rc={rc} required={req.value}")
    return out[: ol.value].tobytes()


@dataclass
class Lz4Result:
    code: int
    written: int
    position: int  # bytes_read (EOF), required (BufferTooSmall), output_pos (offset error)
    provided: int  # `provided` of BufferTooSmall
    data: bytes


def lz4_decompress_block(data, output_size: int, capacity: int | None = None) -> Lz4Result:
    """block.rs:261 decompress_block(input, &mut output[capacity], output_size)."""
    src = _as_u8(data)
    cap = output_size if capacity is None else capacity
    out = np.zeros(max(cap, 1), dtype=np.uint8)
    w, p, a = C.c_size_t(0), C.c_size_t(0), C.c_size_t(0)
    rc = lib().orc_lz4_decompress_block(_u8(src) if src.size else None, src.size, _u8(out), cap,
                                        output_size, C.byref(w), C.byref(p), C.byref(a))
    return Lz4Result(rc, w.value, p.value, a.value, out[: w.value].tobytes() if rc == OK else b"")


BLOCK_DESC = np.dtype([("src_off", "<u8"), ("dst_off", "<u8"), ("src_len", "<u4"),
                       ("dst_cap", "<u4"), ("out_size", "<u4"), ("pad", "<u4")])
BLOCK_STATUS = np.dtype([("code", "<i4"), ("pad", "<i4"), ("position", "<u8"),
                         ("aux", "<u8"), ("written", "<u8")])


def lz4_decompress_batch(src: np.ndarray, descs: np.ndarray, dst_size: int, threads: int = 0):
    """Many independent decompress_block calls (one per descriptor), OpenMP over blocks."""
    src = np.ascontiguousarray(src, dtype=np.uint8)
    descs = np.ascontiguousarray(descs, dtype=BLOCK_DESC)
    dst = np.zeros(max(dst_size, 1), dtype=np.uint8)
    st = np.zeros(len(descs), dtype=BLOCK_STATUS)
    lib().orc_lz4_decompress_batch(_u8(src), descs.ctypes.data, len(descs), _u8(dst),
                                   st.ctypes.data, threads)
    return dst[:dst_size], st


def lz4_compress_chunks(data, block: int = DEFAULT_BLOCK_SIZE, threads: int = 0):
    """HctWriter::compress_data (tensor.rs:556-562): compress `block`-sized chunks.

    Returns (concatenated compressed bytes as np.uint8, per-block lengths u32).
    """
    src = _as_u8(data)
    n = src.size
    nb = 0 if n == 0 else (n + block - 1) // block
    stride = max_compressed_size(block)
    out = np.empty(max(nb * stride, 1), dtype=np.uint8)
    lens = np.zeros(max(nb, 1), dtype=np.uint32)
    rc = lib().orc_lz4_compress_chunks(_u8(src), n, block, _u8(out), stride,
                                       lens.ctypes.data_as(C.POINTER(C.c_uint32)), threads)
    if rc:
        raise RuntimeError("compress_chunks failed")
    lens = lens[:nb]
    if nb == 0:
        return np.zeros(0, np.uint8), lens
    # compact the strided blocks
    offs = np.zeros(nb + 1, dtype=np.int64)
    np.cumsum(lens, out=offs[1:])
    packed = np.empty(int(offs[-1]), dtype=np.uint8)
    view = out[: nb * stride].reshape(nb, stride)
    for i in range(nb):
        packed[offs[i]: offs[i + 1]] = view[i, : lens[i]]
    return packed, lens


# ------------------------------------------------- INT4 (testing/quantization.rs)

def f32_to_f16_bits(v: float) -> int:
    return int(lib().orc_f32_to_f16_bits(float(v)))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().orc_f16_bits_to_f32(int(h)))


def int4_compressed_size(n: int) -> int:
    return int(lib().orc_int4_compressed_size(n))


def quantize_int4(weights) -> bytes:
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
    out = np.zeros(max(int4_compressed_size(w.size), 1), dtype=np.uint8)
    if w.size:
        lib().orc_quantize_int4(_f32(w), w.size, _u8(out))
    return out[: int4_compressed_size(w.size)].tobytes()


def quantize_int4_np(weights) -> np.ndarray:
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
    out = np.zeros(max(int4_compressed_size(w.size), 1), dtype=np.uint8)
    if w.size:
        lib().orc_quantize_int4(_f32(w), w.size, _u8(out))
    return out[: int4_compressed_size(w.size)]


def dequantize_int4(data, num_elements: int) -> np.ndarray:
    src = _as_u8(data)
    out = np.zeros(max(num_elements, 1), dtype=np.float32)
    n = lib().orc_dequantize_int4(_u8(src) if src.size else None, src.size, num_elements, _f32(out))
    return out[:n]


def dequantize_int4_threads(data, num_elements: int, threads: int = 0) -> np.ndarray:
    """dequantize_int4 with OpenMP over 32-element blocks (the CPU baseline)."""
    src = _as_u8(data)
    out = np.empty(max(num_elements, 1), dtype=np.float32)
    n = lib().orc_dequantize_int4_threads(_u8(src) if src.size else None, src.size,
                                          num_elements, _f32(out), threads)
    return out[:n]


def f32_to_f16_rne(x: float) -> int:
    """half::f16::from_f32 bits (IEEE round-to-nearest-even)."""
    return int(lib().orc_f32_to_f16_rne(float(x)))


def quantize_int4_mp(weights) -> bytes:
    """mixed_precision.rs:448-486 (scales as round-to-nearest-even f16)."""
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
    out = np.zeros(max(int4_compressed_size(w.size), 1), dtype=np.uint8)
    if w.size:
        lib().orc_quantize_int4_mp(_f32(w), w.size, _u8(out))
    return out[: int4_compressed_size(w.size)].tobytes()


def dequantize_int4_mp(data, num_elements: int) -> np.ndarray:
    """mixed_precision.rs:489-539 (n values, zero-filled when the data is short)."""
    src = _as_u8(data)
    out = np.zeros(max(num_elements, 1), dtype=np.float32)
    n = lib().orc_dequantize_int4_mp(_u8(src) if src.size else None, src.size, num_elements,
                                     _f32(out))
    return out[:n]


# ------------------------------------------------------------------ DCT (dct.rs)

def dct_1d(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty_like(x)
    lib().orc_dct_1d(_f32(x), _f32(out), x.size)
    return out


def idct_1d(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty_like(x)
    lib().orc_idct_1d(_f32(x), _f32(out), x.size)
    return out


def dct_2d(x: np.ndarray, threads: int = 0) -> np.ndarray:
    """dct.rs:282 dct_2d(input, output, width=cols, height=rows)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    h, w = x.shape
    out = np.empty_like(x)
    lib().orc_dct_2d(_f32(x), _f32(out), w, h, threads)
    return out


def idct_2d(x: np.ndarray, threads: int = 0) -> np.ndarray:
    """dct.rs:311 idct_2d(input, output, width=cols, height=rows)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    h, w = x.shape
    out = np.empty_like(x)
    lib().orc_idct_2d(_f32(x), _f32(out), w, h, threads)
    return out


def idct_2d_f64_truth(x: np.ndarray) -> np.ndarray:
    """Orthonormal DCT-III in float64 (scipy): the truth the f32 paths are held to."""
    import scipy.fft

    return scipy.fft.idctn(np.asarray(x, dtype=np.float64), type=2, norm="ortho")


def dct_2d_f64_truth(x: np.ndarray) -> np.ndarray:
    import scipy.fft

    return scipy.fft.dctn(np.asarray(x, dtype=np.float64), type=2, norm="ortho")


# ------------------------------------------- spectral top-k (compressive.rs:140-172)

def retain_count(n: int, ratio: float) -> int:
    return int(lib().orc_retain_count(n, ratio))


def topk_bitmap(coeffs: np.ndarray, k: int, threads: int = 0) -> np.ndarray:
    c = np.ascontiguousarray(coeffs, dtype=np.float32).reshape(-1)
    bm = np.zeros(max((c.size + 7) // 8, 1), dtype=np.uint8)
    lib().orc_topk_bitmap(_f32(c), c.size, k, _u8(bm), threads)
    return bm[: (c.size + 7) // 8]


def gather_retained(coeffs: np.ndarray, bitmap: np.ndarray) -> np.ndarray:
    c = np.ascontiguousarray(coeffs, dtype=np.float32).reshape(-1)
    k = int(lib().orc_popcount_bytes(_u8(bitmap), bitmap.size))
    vals = np.empty(max(k, 1), dtype=np.float32)
    lib().orc_gather_retained(_f32(c), c.size, _u8(bitmap), _f32(vals))
    return vals[:k]


def scatter_retained(vals: np.ndarray, bitmap: np.ndarray, n: int) -> np.ndarray:
    v = np.ascontiguousarray(vals, dtype=np.float32)
    dense = np.empty(max(n, 1), dtype=np.float32)
    lib().orc_scatter_retained(_f32(v) if v.size else None, v.size, _u8(bitmap), n, _f32(dense))
    return dense[:n]


def popcount(bitmap: np.ndarray) -> int:
    return int(lib().orc_popcount_bytes(_u8(bitmap), bitmap.size))


from .hct import *  # noqa: E402,F401,F403  (container + composite codec)
