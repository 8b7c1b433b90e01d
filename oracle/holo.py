"""HoloTensor container + spectral fragments (CPU oracle side).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): a restatement of
crates/haagenti-hct/src/holotensor.rs for the spectral encoding.

Container (HoloTensorWriter::write, holotensor.rs:1859-1902):
    header    96 bytes (HoloTensorHeader::to_bytes, :515-568; XXH3-64 of
              bytes [0, 88) at 88 when flag 0x0001)
    index     total_fragments x 24 bytes (FragmentIndexEntry, :332-380)
    data      the fragments, concatenated, at data_offset + entry.offset
Reader (HoloTensorReader, :1935-2192): header checks of from_bytes
(:571-656), the inline-fragment form for total_fragments == 0
(:1978-2003), per-fragment XXH3 of the stored bytes when flag 0x0002
(:2069-2077) and zstd when entry flag bit 0 is set (:2081-2091).

Spectral fragments (SpectralEncoder::encode_2d, :734-780): "SV03" raster
slices, fragment f holding the f32 DCT coefficients at raster positions
f, f + F, f + 2F, ... after a 20-byte header
    magic 0x33305653 | num_coeffs | num_fragments | slice_offset | slice_count
SpectralDecoder (:806-1066) writes them into an accumulator (later
fragments overwrite), quality = covered positions / n, and reconstructs with
idct_2d(width = cols, height = rows).  The decoder's 2-D view of the header
shape is HoloTensorDecoder::new's (:1732-1759).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from . import dct_2d, idct_2d
from .hct import xxh3_64

HOLO_MAGIC = b"HTNS"
HOLO_VERSION = 1
HOLO_FLAG_HEADER_CHECKSUM = 0x0001
HOLO_FLAG_FRAGMENT_CHECKSUMS = 0x0002
HOLO_FLAG_QUANTIZATION = 0x0004
HOLO_HEADER_SIZE = 96
INDEX_ENTRY_SIZE = 24
ENC_SPECTRAL, ENC_RPH, ENC_LRDF = 0, 1, 2
ALGO_LZ4, ALGO_ZSTD = 0, 1
DTYPE_F32 = 0
SV03_MAGIC = 0x33305653
SV02_MAGIC = 0x32305653

# HolographicEncoding::default_quality_curve (holotensor.rs:111-132):
# (coefficients, min_fragments, sufficient_fragments)
DEFAULT_CURVES = {
    ENC_SPECTRAL: ((0.6, 0.3, 0.08, 0.02), 1, 6),
    ENC_RPH: ((0.1, 0.8, 0.08, 0.02), 2, 6),
    ENC_LRDF: ((0.3, 0.5, 0.15, 0.05), 1, 4),
}


class HoloError(Exception):
    """haagenti_core::Error::CorruptedData raised by the reference."""


@dataclass
class HoloHeader:
    encoding: int = ENC_SPECTRAL
    compression: int = ALGO_ZSTD  # HoloTensorHeader::new's default (:455)
    flags: int = HOLO_FLAG_HEADER_CHECKSUM | HOLO_FLAG_FRAGMENT_CHECKSUMS
    total_fragments: int = 8
    min_fragments: int = 1
    original_size: int = 0
    seed: int = 0
    dtype: int = DTYPE_F32
    shape: list = field(default_factory=list)
    curve: tuple = (0.6, 0.3, 0.08, 0.02)


def f32(x) -> float:
    return float(np.float32(x))


def curve_predict(curve, min_fragments: int, k: int, n: int) -> float:
    """QualityCurve::predict (holotensor.rs:199-220), in f32 arithmetic."""
    if n == 0:
        return 0.0
    if k >= n:
        return 1.0
    if k < min_fragments:
        return 0.0
    x = np.float32(k) / np.float32(n)
    result = np.float32(0.0)
    xp = np.float32(1.0)
    for c in curve:
        result = np.float32(result + np.float32(c) * xp)
        xp = np.float32(xp * x)
    return float(min(max(result, np.float32(0.0)), np.float32(1.0)))


def header_to_bytes(h: HoloHeader) -> bytes:
    """HoloTensorHeader::to_bytes (holotensor.rs:515-568)."""
    b = bytearray()
    b += HOLO_MAGIC
    b += struct.pack("<IBBHHHQQBB", HOLO_VERSION, h.encoding, h.compression, h.flags,
                     h.total_fragments, h.min_fragments, h.original_size, h.seed, h.dtype,
                     len(h.shape))
    for i in range(4):
        b += struct.pack("<Q", h.shape[i] if i < len(h.shape) else 0)
    b += struct.pack("<4f", *h.curve)
    b += bytes(6)
    b += struct.pack("<Q", xxh3_64(bytes(b)))
    assert len(b) == HOLO_HEADER_SIZE
    return bytes(b)


def header_from_bytes(b: bytes) -> HoloHeader:
    """HoloTensorHeader::from_bytes (holotensor.rs:571-656)."""
    if len(b) < HOLO_HEADER_SIZE:
        raise HoloError("header too short")
    if b[0:4] != HOLO_MAGIC:
        raise HoloError("invalid magic bytes")
    version = struct.unpack_from("<I", b, 4)[0]
    if version != HOLO_VERSION:
        raise HoloError(f"unsupported version: {version}")
    flags = struct.unpack_from("<H", b, 10)[0]
    if flags & HOLO_FLAG_HEADER_CHECKSUM:
        if struct.unpack_from("<Q", b, 88)[0] != xxh3_64(b[0:88]):
            raise HoloError("header checksum mismatch")
    if b[8] > 2:
        raise HoloError(f"unknown encoding: {b[8]}")
    if b[9] > 1:
        raise HoloError(f"unknown algorithm: {b[9]}")
    total, minf = struct.unpack_from("<HH", b, 12)
    orig, seed = struct.unpack_from("<QQ", b, 16)
    if b[32] > 4:
        raise HoloError(f"unknown dtype: {b[32]}")
    ndim = b[33]
    if 34 + 8 * ndim > HOLO_HEADER_SIZE:  # the Rust slice would run past the header
        raise HoloError("shape runs past the header")
    shape = [struct.unpack_from("<Q", b, 34 + 8 * i)[0] for i in range(ndim)]
    curve = struct.unpack_from("<4f", b, 66)
    return HoloHeader(b[8], b[9], flags, total, minf, orig, seed, b[32], shape, curve)


def index_entry_bytes(index, flags, offset, csize, usize, checksum) -> bytes:
    """FragmentIndexEntry::to_bytes (holotensor.rs:352-361)."""
    return struct.pack("<HHIIIQ", index, flags, offset, csize, usize, checksum)


def write_holotensor(h: HoloHeader, fragments) -> bytes:
    """HoloTensorWriter::write (holotensor.rs:1859-1902); fragments are
    (index, flags, data) and are stored as given."""
    out = bytearray(header_to_bytes(h))
    off = 0
    for idx, fl, data in fragments:
        out += index_entry_bytes(idx, fl, off, len(data), len(data), xxh3_64(data))
        off += len(data)
    for _, _, data in fragments:
        out += data
    return bytes(out)


def matrix_dims(shape) -> tuple[int, int]:
    """HoloTensorDecoder::new / HoloTensorEncoder::flatten_shape
    (holotensor.rs:1626-1638, 1732-1744): (rows, cols)."""
    if len(shape) == 0:
        return 1, 1
    if len(shape) == 1:
        return 1, int(shape[0])
    if len(shape) == 2:
        return int(shape[0]), int(shape[1])
    return int(shape[0]), int(np.prod([int(d) for d in shape[1:]]))


def sv03_fragments(coeffs: np.ndarray, num_fragments: int) -> list:
    """SpectralEncoder::encode_2d's fragment bodies (holotensor.rs:754-776)
    from the raster-order coefficients."""
    c = np.ascontiguousarray(coeffs, dtype=np.float32).ravel()
    n = c.size
    out = []
    for f in range(num_fragments):
        count = (max(n - f, 0) + num_fragments - 1) // num_fragments
        body = struct.pack("<5I", SV03_MAGIC, n, num_fragments, f, count)
        out.append(body + c[f::num_fragments].tobytes())
    return out


def encode_spectral(w: np.ndarray, shape=None, num_fragments: int = 8, seed: int = 0,
                    compression: int = ALGO_LZ4, coeffs=None) -> bytes:
    """HoloTensorEncoder(Spectral).encode_nd + HoloTensorWriter::write
    (holotensor.rs:1563-1571, 1656-1688, 1859-1902): the encoder's defaults
    (8 fragments, seed 0, LZ4 in the header), fragments stored uncompressed
    as the writer stores them."""
    shape = list(w.shape) if shape is None else list(shape)
    rows, cols = matrix_dims(shape)
    if coeffs is None:
        coeffs = dct_2d(np.ascontiguousarray(w, dtype=np.float32).reshape(rows, cols))
    curve, minf, _ = DEFAULT_CURVES[ENC_SPECTRAL]
    h = HoloHeader(ENC_SPECTRAL, compression, HOLO_FLAG_HEADER_CHECKSUM |
                   HOLO_FLAG_FRAGMENT_CHECKSUMS, num_fragments, minf,
                   rows * cols * 4, seed, DTYPE_F32, [int(d) for d in shape], curve)
    frags = sv03_fragments(coeffs, num_fragments)
    return write_holotensor(h, [(i, 0, d) for i, d in enumerate(frags)])


@dataclass
class ParsedHolo:
    header: HoloHeader
    entries: list  # (index, flags, offset, csize, usize, checksum)
    data_offset: int
    inline: bool
    file: bytes


def parse_holotensor(file: bytes) -> ParsedHolo:
    """HoloTensorReader::new (holotensor.rs:1948-2011)."""
    h = header_from_bytes(file[:HOLO_HEADER_SIZE])
    n = h.total_fragments
    if len(file) < HOLO_HEADER_SIZE + n * INDEX_ENTRY_SIZE:
        raise HoloError("failed to read fragment index")
    entries = [struct.unpack_from("<HHIIIQ", file, HOLO_HEADER_SIZE + i * INDEX_ENTRY_SIZE)
               for i in range(n)]
    data_offset = HOLO_HEADER_SIZE + n * INDEX_ENTRY_SIZE
    inline = False
    if n == 0 and len(file) >= data_offset + INDEX_ENTRY_SIZE:
        e = struct.unpack_from("<HHIIIQ", file, data_offset)
        if e[0] == 0 and 0 < e[3] < 1_000_000_000:
            entries = [e]
            inline = True
    return ParsedHolo(h, entries, data_offset, inline, file)


def total_fragments(p: ParsedHolo) -> int:
    return 1 if p.inline else p.header.total_fragments


def read_fragment(p: ParsedHolo, i: int):
    """HoloTensorReader::read_fragment (holotensor.rs:2039-2098): the entry
    whose index is i, checksum of the stored bytes, zstd when flag bit 0."""
    if p.inline:
        if i != 0:
            raise HoloError(f"inline format only has fragment 0, requested {i}")
        e = p.entries[0]
        start = p.data_offset + INDEX_ENTRY_SIZE + e[2]
    else:
        e = next((x for x in p.entries if x[0] == i), None)
        if e is None:
            raise HoloError(f"fragment {i} not found")
        start = p.data_offset + e[2]
    data = p.file[start:start + e[3]]
    if len(data) < e[3]:
        raise HoloError("failed to read fragment data")
    if p.header.flags & HOLO_FLAG_FRAGMENT_CHECKSUMS and xxh3_64(data) != e[5]:
        raise HoloError(f"fragment {i} checksum mismatch")
    if e[1] & 1:  # zstd::decode_all, i.e. libzstd (oracle/zstd_ref.py)
        from . import zstd_ref

        ok, dec = zstd_ref.decompress(data, max(e[4], 1 << 26))
        if not ok:
            raise HoloError(f"failed to decompress fragment {i}: {dec}")
        data = dec
    return e[0], data


def fragments_for_quality(p: ParsedHolo, target: float) -> int:
    """How many fragments HoloTensorReader::read_to_quality reads
    (holotensor.rs:2164-2187)."""
    total = total_fragments(p)
    h = p.header
    for i in range(total):
        if curve_predict(h.curve, h.min_fragments, i + 1, max(total, 1)) >= target:
            return i + 1
    return total


class SpectralDecoderCpu:
    """SpectralDecoder restricted to SV03 fragments (holotensor.rs:806-1066)."""

    def __init__(self, rows: int, cols: int):
        self.rows, self.cols = rows, cols
        self.acc = np.zeros(rows * cols, np.float32)
        self.set = np.zeros(rows * cols, bool)
        self.loaded = 0

    def add_fragment(self, data: bytes):
        """add_fragment + add_fragment_v3 (holotensor.rs:840-858, 979-1015)."""
        if len(data) < 8:
            raise HoloError("fragment too short")
        magic = struct.unpack_from("<I", data, 0)[0]
        if magic != SV03_MAGIC:
            raise NotImplementedError("V1/V2 spectral fragment")
        if len(data) < 20:
            raise HoloError("V3 fragment too short")
        num_coeffs, F, start, _count = struct.unpack_from("<4I", data, 4)
        nv = (len(data) - 20) // 4
        vals = np.frombuffer(data, np.float32, count=nv, offset=20)
        n = self.acc.size
        if F == 0:
            if start < num_coeffs and nv and start < n:
                self.acc[start] = vals[-1]
                self.set[start] = True
        else:
            cnt = min(nv, (num_coeffs - start + F - 1) // F if start < num_coeffs else 0)
            pos = start + F * np.arange(cnt, dtype=np.int64)
            keep = pos < n
            self.acc[pos[keep]] = vals[:cnt][keep]
            self.set[pos[keep]] = True
        self.loaded += 1

    def quality(self) -> float:
        return float(np.float32(np.count_nonzero(self.set)) / np.float32(self.acc.size))

    def reconstruct(self) -> np.ndarray:
        return idct_2d(self.acc.reshape(self.rows, self.cols))


def decode_cpu(file: bytes, num_fragments=None):
    """read fragments 0..k-1 into a SpectralDecoder and reconstruct (the
    steps of decode_from_file / decode_from_file_progressive,
    holotensor.rs:2310-2357).  Returns (rows x cols f32, decoder quality)."""
    p = parse_holotensor(file)
    if p.header.encoding != ENC_SPECTRAL:
        raise NotImplementedError("non-spectral HoloTensor encoding")
    rows, cols = matrix_dims(p.header.shape)
    dec = SpectralDecoderCpu(rows, cols)
    k = total_fragments(p) if num_fragments is None else num_fragments
    for i in range(k):
        dec.add_fragment(read_fragment(p, i)[1])
    if dec.loaded == 0:
        raise HoloError("no fragments loaded")
    return dec.reconstruct(), dec.quality()
