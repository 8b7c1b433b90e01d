"""Writer side: encode tensors into the HCT files the GPU decoder reads.

Counterparts of the reference's encoder-side functions (not timed; they make
the decoder's inputs):

* ``quantize_int4`` -- crates/haagenti/src/testing/quantization.rs:30-70,
  vectorised: per 32-element block scale = max|x| / 7 (1.0 if <= 1e-10),
  stored as the reference's truncating, flush-to-zero f16; q = x / scale
  rounded half away from zero, saturated to i8, clamped to [-8, 7], stored
  as nibble q + 8, low nibble first.
* ``spectral_select`` -- CompressiveSpectralEncoder::encode_2d's retention
  (crates/haagenti/src/compressive.rs:140-172): keep the
  ``((n as f32 * ratio) as usize).max(1)`` largest |coefficients|, ties to
  the lower index, bitmap LSB-first, values in ascending index order.
* ``write_hct`` -- HctWriter / HctWriterV2 (crates/haagenti-hct/src/tensor.rs:
  519-617, 679-829) with LZ4 blocks from the library's compress_block port.
* ``encode_spectral_q4`` -- this library's composite payload
  (bitmap ++ INT4 of the retained DCT coefficients, flag 0x0100).

The forward DCT uses scipy's single-precision orthonormal DCT-II
(``scipy.fft.dctn(type=2, norm="ortho")``), the same transform as
haagenti_core::dct::dct_2d (crates/haagenti-core/src/dct.rs:282-308).
"""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

from . import _lib as L

DEFAULT_BLOCK_SIZE = 16 * 1024
ALGO_LZ4 = 0
DTYPE_I4 = 4
FLAG_HEADER_CHECKSUM, FLAG_BLOCK_CHECKSUMS = 0x0001, 0x0002
FLAG_SPECTRAL_Q4 = L.FLAG_SPECTRAL_Q4


def _f32_to_f16_trunc(v: np.ndarray) -> np.ndarray:
    """quantization.rs:136-163, element-wise on f32 arrays -> u16 bits."""
    b = np.ascontiguousarray(v, np.float32).view(np.uint32)
    sign = (b >> 31) & 1
    exp = ((b >> 23) & 0xFF).astype(np.int32)
    frac = b & 0x7FFFFF
    ne = exp - 127 + 15
    out = (sign << 15).astype(np.uint32)
    inf_nan = exp == 0xFF
    out = np.where(inf_nan, (sign << 15) | (0x1F << 10) | (frac >> 13), out)
    normal = (exp != 0) & ~inf_nan
    over = normal & (ne >= 31)
    out = np.where(over, (sign << 15) | (0x1F << 10), out)
    ok = normal & (ne > 0) & (ne < 31)
    out = np.where(ok, (sign << 15) | (np.clip(ne, 0, 31).astype(np.uint32) << 10) | (frac >> 13), out)
    return out.astype(np.uint16)


def int4_compressed_size(n: int) -> int:
    return 0 if n == 0 else ((n + 31) // 32) * 2 + (n + 1) // 2


def quantize_int4(weights) -> np.ndarray:
    """quantization.rs:30-70 via the library's OpenMP port (hct_b200_quantize_int4)."""
    w = np.ascontiguousarray(weights, np.float32).reshape(-1)
    out = np.zeros(max(int4_compressed_size(w.size), 1), np.uint8)
    if w.size:
        rc = L.load().hct_b200_quantize_int4(w.ctypes.data, w.size, out.ctypes.data)
        if rc:
            raise RuntimeError(f"quantize_int4 failed: {rc}")
    return out[: int4_compressed_size(w.size)]


def quantize_int4_mp(weights) -> np.ndarray:
    """mixed_precision.rs:448-486 (round-to-nearest-even f16 scales) via
    hct_b200_quantize_int4_mp."""
    w = np.ascontiguousarray(weights, np.float32).reshape(-1)
    out = np.zeros(max(int4_compressed_size(w.size), 1), np.uint8)
    if w.size:
        rc = L.load().hct_b200_quantize_int4_mp(w.ctypes.data, w.size, out.ctypes.data)
        if rc:
            raise RuntimeError(f"quantize_int4_mp failed: {rc}")
    return out[: int4_compressed_size(w.size)]


def retain_count(n: int, ratio: float) -> int:
    p = np.float32(n) * np.float32(ratio)
    return max(int(p) if p > 0 else 0, 1)


def spectral_select(coeffs: np.ndarray, ratio: float = 0.30):
    """Returns (bitmap u8, retained values f32 in index order)."""
    c = np.ascontiguousarray(coeffs, np.float32).reshape(-1)
    n = c.size
    k = min(retain_count(n, ratio), n)
    bitmap = np.zeros(max((n + 7) // 8, 1), np.uint8)
    vals = np.empty(max(k, 1), np.float32)
    cnt = C.c_size_t(0)
    rc = L.load().hct_b200_spectral_select(c.ctypes.data, n, k, bitmap.ctypes.data,
                                           vals.ctypes.data, C.byref(cnt))
    if rc:
        raise RuntimeError(f"spectral_select failed: {rc}")
    return bitmap[: (n + 7) // 8], vals[: cnt.value]


def lz4_compress_chunks(data, block_size: int = DEFAULT_BLOCK_SIZE):
    """Compress block_size chunks with the library's compress_block port."""
    src = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    n = src.size
    nb = 0 if n == 0 else (n + block_size - 1) // block_size
    lib = L.load()
    stride = int(lib.hct_b200_lz4_max_compressed_size(block_size))
    out = np.empty(max(nb * stride, 1), np.uint8)
    lens = np.zeros(max(nb, 1), np.uint32)
    rc = lib.hct_b200_lz4_compress_chunks(src.ctypes.data, n, block_size, out.ctypes.data, stride,
                                          lens.ctypes.data_as(C.POINTER(C.c_uint32)))
    if rc:
        raise RuntimeError(f"compress_chunks failed: {rc}")
    lens = lens[:nb]
    if nb == 0:
        return np.zeros(0, np.uint8), lens
    view = out[: nb * stride].reshape(nb, stride)
    mask = np.arange(stride)[None, :] < lens[:, None]
    return view[mask], lens


def _xxh3(data) -> int:
    import xxhash

    return xxhash.xxh3_64_intdigest(data)


def write_hct(payload, shape, dtype: int = DTYPE_I4, flags: int = 0, version: int = 1,
              block_size: int = DEFAULT_BLOCK_SIZE) -> bytes:
    """HCT v1/v2 file bytes: header, (v2: XXH3 checksums), block index, LZ4 blocks."""
    payload = np.ascontiguousarray(payload).view(np.uint8).reshape(-1)
    comp, lens = lz4_compress_chunks(payload, block_size)
    nb = len(lens)
    offs = np.zeros(nb, np.uint64)
    if nb:
        offs[1:] = np.cumsum(lens[:-1], dtype=np.uint64)
    if version >= 2:
        flags |= FLAG_HEADER_CHECKSUM | FLAG_BLOCK_CHECKSUMS
    hdr = bytearray(64)
    hdr[0:4] = b"HCTN"
    struct.pack_into("<IBBHQQII", hdr, 4, version, ALGO_LZ4, dtype, flags, payload.size,
                     comp.size, block_size, nb)
    hdr[36] = len(shape)
    for i, d in enumerate(list(shape)[:4]):
        struct.pack_into("<Q", hdr, 37 + 8 * i, int(d))
    if version >= 2:
        struct.pack_into("<Q", hdr, 56, _xxh3(bytes(hdr[:56])))
        idx = np.zeros(nb, dtype=[("off", "<u4"), ("len", "<u4"), ("xxh", "<u8")])
        starts = np.concatenate([[0], np.cumsum(lens, dtype=np.int64)])
        idx["xxh"] = [_xxh3(comp[starts[i]:starts[i + 1]].tobytes()) for i in range(nb)]
    else:
        idx = np.zeros(nb, dtype=[("off", "<u4"), ("len", "<u4")])
    idx["off"] = offs.astype(np.uint32)
    idx["len"] = lens
    return b"".join([bytes(hdr), idx.tobytes(), comp.tobytes()])


def dct_2d(w: np.ndarray, workers: int = -1) -> np.ndarray:
    import scipy.fft

    return scipy.fft.dctn(np.ascontiguousarray(w, np.float32), type=2, norm="ortho",
                          workers=workers).astype(np.float32, copy=False)


def tensor_dims(shape) -> tuple[int, int]:
    shape = [int(s) for s in shape]
    if len(shape) == 1:
        return 1, shape[0]
    return int(np.prod(shape[:-1])), shape[-1]


def encode_spectral_q4(w: np.ndarray, retention: float = 0.30, version: int = 1,
                       block_size: int = DEFAULT_BLOCK_SIZE, coeffs: np.ndarray | None = None) -> bytes:
    """W -> orthonormal DCT-II -> top-k bitmap -> INT4 of retained values -> LZ4 HCT."""
    m, n = tensor_dims(w.shape)
    if coeffs is None:
        coeffs = dct_2d(np.asarray(w, np.float32).reshape(m, n))
    bitmap, vals = spectral_select(coeffs, retention)
    payload = np.concatenate([bitmap, quantize_int4(vals)])
    return write_hct(payload, list(w.shape), DTYPE_I4, FLAG_SPECTRAL_Q4, version, block_size)


def encode_hct_v3(w: np.ndarray, retention: float = 0.30, num_fragments: int = 1,
                  coeffs: np.ndarray | None = None) -> bytes:
    """HCT V3 fragment container (the layout crates/haagenti-cuda/src/decompress.rs:322-438
    parses): DCT-II -> top-k -> fp16 values (round to nearest even), the retained set
    split in index order over ``num_fragments`` fragments with disjoint bitmaps."""
    m, n = tensor_dims(w.shape)
    if coeffs is None:
        coeffs = dct_2d(np.asarray(w, np.float32).reshape(m, n))
    bitmap, vals = spectral_select(coeffs, retention)
    total = m * n
    idx = np.nonzero(np.unpackbits(bitmap, bitorder="little")[:total])[0]
    out = [struct.pack("<H", num_fragments)]
    for f, (part, pv) in enumerate(zip(np.array_split(idx, num_fragments),
                                       np.array_split(vals, num_fragments))):
        fb = np.zeros((total + 7) // 8, np.uint8)
        np.bitwise_or.at(fb, part // 8, (1 << (part % 8)).astype(np.uint8))
        data = struct.pack("<I", part.size) + fb.tobytes() + pv.astype(np.float16).tobytes()
        out.append(struct.pack("<HHQI", f, 0, _xxh3(data), len(data)))
        out.append(data)
    return b"".join(out)


_ZSTD = None


def zstd_compress(data, level: int = 3, checksum: bool = False) -> bytes:
    """One zstd frame of ``data`` from the system libzstd (the writer side of
    the zstd-compressed fragments and containers the GPU decoder reads; the
    reference writes them with the `zstd` crate, i.e. libzstd)."""
    global _ZSTD
    if _ZSTD is None:
        lib = C.CDLL("libzstd.so.1")
        lib.ZSTD_createCCtx.restype = C.c_void_p
        lib.ZSTD_freeCCtx.argtypes = [C.c_void_p]
        lib.ZSTD_CCtx_setParameter.restype = C.c_size_t
        lib.ZSTD_CCtx_setParameter.argtypes = [C.c_void_p, C.c_int, C.c_int]
        lib.ZSTD_compressBound.restype = C.c_size_t
        lib.ZSTD_compressBound.argtypes = [C.c_size_t]
        lib.ZSTD_compress2.restype = C.c_size_t
        lib.ZSTD_compress2.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        lib.ZSTD_isError.restype = C.c_uint
        lib.ZSTD_isError.argtypes = [C.c_size_t]
        _ZSTD = lib
    lib = _ZSTD
    src = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray)
                               else data.view(np.uint8).reshape(-1))
    cctx = lib.ZSTD_createCCtx()
    try:
        lib.ZSTD_CCtx_setParameter(cctx, 100, int(level))      # ZSTD_c_compressionLevel
        lib.ZSTD_CCtx_setParameter(cctx, 201, int(checksum))   # ZSTD_c_checksumFlag
        cap = lib.ZSTD_compressBound(src.size) + 64
        out = np.empty(cap, np.uint8)
        n = lib.ZSTD_compress2(cctx, out.ctypes.data, cap, src.ctypes.data if src.size else None,
                               src.size)
        if lib.ZSTD_isError(n):
            raise ValueError("zstd compression failed")
        return out[:n].tobytes()
    finally:
        lib.ZSTD_freeCCtx(cctx)


HOLO_SPECTRAL_CURVE = (0.6, 0.3, 0.08, 0.02)  # holotensor.rs:114-118


def holo_dims(shape) -> tuple[int, int]:
    """HoloTensorEncoder::flatten_shape (holotensor.rs:1626-1638)."""
    shape = [int(s) for s in shape]
    if len(shape) == 0:
        return 1, 1
    if len(shape) == 1:
        return 1, shape[0]
    return shape[0], int(np.prod(shape[1:]))


def encode_holotensor(w: np.ndarray, num_fragments: int = 8, shape=None, seed: int = 0,
                      coeffs: np.ndarray | None = None) -> bytes:
    """Spectral HoloTensor file (HoloTensorEncoder::encode_nd + HoloTensorWriter::write,
    crates/haagenti-hct/src/holotensor.rs:1656-1688, 1859-1902): the DCT-II
    coefficients dealt out in raster order to ``num_fragments`` "SV03" fragments
    (fragment f holds positions f, f + F, ...), header and fragment checksums on."""
    shape = list(w.shape) if shape is None else [int(d) for d in shape]
    rows, cols = holo_dims(shape)
    if coeffs is None:
        coeffs = dct_2d(np.asarray(w, np.float32).reshape(rows, cols))
    c = np.ascontiguousarray(coeffs, np.float32).reshape(-1)
    n, F = c.size, max(int(num_fragments), 1)
    hdr = bytearray(b"HTNS")
    hdr += struct.pack("<IBBHHHQQBB", 1, 0, 0, 0x0003, F, 1, n * 4, seed, 0, len(shape))
    for i in range(4):
        hdr += struct.pack("<Q", shape[i] if i < len(shape) else 0)
    hdr += struct.pack("<4f", *HOLO_SPECTRAL_CURVE) + bytes(6)
    hdr += struct.pack("<Q", _xxh3(bytes(hdr)))
    frags = []
    for f in range(F):
        count = (max(n - f, 0) + F - 1) // F
        frags.append(struct.pack("<5I", 0x33305653, n, F, f, count) + c[f::F].tobytes())
    index, off = [], 0
    for f, d in enumerate(frags):
        index.append(struct.pack("<HHIIIQ", f, 0, off, len(d), len(d), _xxh3(d)))
        off += len(d)
    return b"".join([bytes(hdr)] + index + frags)


def encode_int4(w: np.ndarray, version: int = 1, block_size: int = DEFAULT_BLOCK_SIZE) -> bytes:
    """INT4 + LZ4 on raw weights (examples/safetensors_to_int4_hct.rs:241-284)."""
    return write_hct(quantize_int4(w), list(w.shape), DTYPE_I4, 0, version, block_size)


GEN_CHUNK = 1 << 22


def synthetic_weight(shape, seed: int, outlier_frac: float = 0.01, std: float = 0.02) -> np.ndarray:
    """Seeded N(0, std) f32 weights with a seeded 1% of columns scaled x10.

    The flattened tensor is filled in 2^22-element chunks, chunk i from
    PCG64(SeedSequence(seed).spawn(n)[i]) standard normals (chunks in
    parallel threads); outlier columns are the first 1% of a permutation
    drawn from default_rng([seed, 1]).
    """
    from concurrent.futures import ThreadPoolExecutor

    shape = tuple(int(s) for s in shape)
    n = int(np.prod(shape))
    w = np.empty(n, np.float32)
    nch = max(1, (n + GEN_CHUNK - 1) // GEN_CHUNK)
    seqs = np.random.SeedSequence(seed).spawn(nch)

    def fill(i):
        a, b = i * GEN_CHUNK, min(n, (i + 1) * GEN_CHUNK)
        np.random.Generator(np.random.PCG64(seqs[i])).standard_normal(
            out=w[a:b], dtype=np.float32)
        w[a:b] *= np.float32(std)

    with ThreadPoolExecutor(max_workers=min(nch, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, range(nch)))
    w = w.reshape(shape)
    if outlier_frac > 0 and len(shape) == 2:
        nout = max(1, int(shape[1] * outlier_frac))
        cols = np.random.default_rng([seed, 1]).permutation(shape[1])[:nout]
        w[:, cols] *= np.float32(10.0)
    return w
