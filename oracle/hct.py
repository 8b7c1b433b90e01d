"""HCT container + composite spectral INT4 codec (CPU oracle side).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Container: crates/haagenti-hct/src/tensor.rs
  * 64-byte header (HctHeader::to_bytes, tensor.rs:297-329; v2 header written by
    HctWriterV2::finish, tensor.rs:764-795, XXH3-64 over bytes [0,56) at 56),
  * optional 8-byte QuantizationMetadata (tensor.rs:181-212),
  * block index: 8 bytes (offset u32, compressed_size u32, tensor.rs:379-405)
    or 16 bytes with an XXH3-64 of the compressed block (tensor.rs:232-271),
  * concatenated LZ4 blocks of `block_size` uncompressed bytes
    (HctWriter::compress_data, tensor.rs:556-562).

Composite spectral payload ("HCT-Q4", defined by this project, flag 0x0100):
    payload = bitmap[ceil(M*N/8)]            (compressive.rs:157-163, LSB first)
            ++ quantize_int4(values)          (quantization.rs:30-70)
    values  = dct_2d(W)[i] for set bits i in ascending order (compressive.rs:167-172)
    shape   = [M, N] (rows, cols); dtype = I4; algorithm = LZ4.
Decode: LZ4 -> dequantize_int4 -> scatter by bitmap rank -> idct_2d(width=N, height=M).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from . import (BLOCK_DESC, DEFAULT_BLOCK_SIZE, dct_2d, dequantize_int4, gather_retained,
               idct_2d, lz4_compress_chunks, lz4_decompress_batch, popcount,
               quantize_int4_np, retain_count, scatter_retained, topk_bitmap)

HCT_MAGIC = b"HCTN"
HCT_VERSION = 1
HCT_VERSION_V2 = 2
FLAG_HEADER_CHECKSUM = 0x0001
FLAG_BLOCK_CHECKSUMS = 0x0002
FLAG_QUANTIZATION = 0x0004
FLAG_TENSOR_NAME = 0x0008
FLAG_HOLOGRAPHIC = 0x0010
FLAG_SPECTRAL_Q4 = 0x0100  # this project's composite payload (not a reference flag)

ALGO_LZ4, ALGO_ZSTD = 0, 1
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I8, DTYPE_I4 = 0, 1, 2, 3, 4


def xxh3_64(data) -> int:
    import xxhash

    return xxhash.xxh3_64_intdigest(bytes(data))


@dataclass
class HctHeader:
    algorithm: int = ALGO_LZ4
    dtype: int = DTYPE_I4
    flags: int = 0
    original_size: int = 0
    compressed_size: int = 0
    block_size: int = DEFAULT_BLOCK_SIZE
    num_blocks: int = 0
    shape: list = field(default_factory=list)
    version: int = HCT_VERSION

    def to_bytes(self) -> bytes:
        buf = bytearray(64)
        buf[0:4] = HCT_MAGIC
        struct.pack_into("<IBBHQQII", buf, 4, self.version, self.algorithm, self.dtype,
                         self.flags, self.original_size, self.compressed_size,
                         self.block_size, self.num_blocks)
        buf[36] = len(self.shape)
        for i, d in enumerate(self.shape[:4]):
            struct.pack_into("<Q", buf, 37 + 8 * i, int(d))
        if self.version >= HCT_VERSION_V2:
            struct.pack_into("<Q", buf, 56, xxh3_64(bytes(buf[:56])))
        return bytes(buf)

    @staticmethod
    def from_bytes(buf: bytes) -> "HctHeader":
        if buf[0:4] != HCT_MAGIC:
            raise ValueError("invalid HCT magic")
        version, algo, dtype, flags, orig, comp, bsz, nb = struct.unpack_from("<IBBHQQII", buf, 4)
        rank = buf[36]
        shape = [struct.unpack_from("<Q", buf, 37 + 8 * i)[0] for i in range(min(rank, 4))]
        return HctHeader(algo, dtype, flags, orig, comp, bsz, nb, shape, version)


def write_hct(payload, shape, dtype: int = DTYPE_I4, flags: int = 0, version: int = 1,
              block_size: int = DEFAULT_BLOCK_SIZE, block_checksums: bool = True,
              quant_meta: bytes | None = None, threads: int = 0) -> bytes:
    """HctWriter / HctWriterV2 (tensor.rs:519-617, 679-829) with LZ4 blocks."""
    payload = np.ascontiguousarray(payload).view(np.uint8).reshape(-1)
    comp, lens = lz4_compress_chunks(payload, block_size, threads)
    nb = len(lens)
    offs = np.zeros(nb, dtype=np.uint64)
    if nb:
        offs[1:] = np.cumsum(lens[:-1], dtype=np.uint64)
    if version >= HCT_VERSION_V2:
        flags |= FLAG_HEADER_CHECKSUM
        if block_checksums:
            flags |= FLAG_BLOCK_CHECKSUMS
        if quant_meta is not None:
            flags |= FLAG_QUANTIZATION
    hdr = HctHeader(ALGO_LZ4, dtype, flags, int(payload.size), int(comp.size), block_size, nb,
                    list(shape), version)
    parts = [np.frombuffer(hdr.to_bytes(), np.uint8)]
    if version >= HCT_VERSION_V2 and quant_meta is not None:
        parts.append(np.frombuffer(quant_meta, np.uint8))
    if version >= HCT_VERSION_V2 and block_checksums:
        idx = np.zeros(nb, dtype=[("off", "<u4"), ("len", "<u4"), ("xxh", "<u8")])
        idx["off"] = offs.astype(np.uint32)
        idx["len"] = lens
        start = 0
        sums = np.zeros(nb, dtype=np.uint64)
        for i in range(nb):
            sums[i] = xxh3_64(comp[start: start + lens[i]].tobytes())
            start += int(lens[i])
        idx["xxh"] = sums
    else:
        idx = np.zeros(nb, dtype=[("off", "<u4"), ("len", "<u4")])
        idx["off"] = offs.astype(np.uint32)
        idx["len"] = lens
    parts.append(idx.view(np.uint8).reshape(-1))
    parts.append(comp)
    return np.concatenate(parts).tobytes()


@dataclass
class ParsedHct:
    header: HctHeader
    offsets: np.ndarray
    sizes: np.ndarray
    checksums: np.ndarray | None
    data: np.ndarray  # compressed data section
    quant_meta: bytes | None

    def expected_size(self, i: int) -> int:
        """HctReader::decompress_block expected size (tensor.rs:494-500)."""
        nb = len(self.sizes)
        if i == nb - 1:
            return self.header.original_size - (nb - 1) * self.header.block_size
        return self.header.block_size


def parse_hct(file: bytes, validate: bool = True) -> ParsedHct:
    """HctReader::new / HctReaderV2::new (tensor.rs:417-444, 841-922)."""
    buf = np.frombuffer(file, dtype=np.uint8)
    hdr = HctHeader.from_bytes(file[:64])
    pos = 64
    qm = None
    if hdr.version >= HCT_VERSION_V2 and hdr.flags & FLAG_HEADER_CHECKSUM and validate:
        stored = struct.unpack_from("<Q", file, 56)[0]
        if xxh3_64(file[:56]) != stored:
            raise ValueError("header checksum mismatch")
    if hdr.flags & FLAG_QUANTIZATION and hdr.version >= HCT_VERSION_V2:
        qm = file[pos: pos + 8]
        pos += 8
    with_sums = hdr.version >= HCT_VERSION_V2 and bool(hdr.flags & FLAG_BLOCK_CHECKSUMS)
    ent = 16 if with_sums else 8
    nb = hdr.num_blocks
    idx = buf[pos: pos + nb * ent]
    pos += nb * ent
    if with_sums:
        rec = idx.view([("off", "<u4"), ("len", "<u4"), ("xxh", "<u8")])
        sums = rec["xxh"].copy()
    else:
        rec = idx.view([("off", "<u4"), ("len", "<u4")])
        sums = None
    return ParsedHct(hdr, rec["off"].astype(np.uint64), rec["len"].astype(np.uint32), sums,
                     buf[pos:], qm)


def decompress_all_cpu(p: ParsedHct, threads: int = 0, validate: bool = True) -> np.ndarray:
    """HctReader::decompress_all with Lz4Decompressor (tensor.rs:506-515)."""
    nb = len(p.sizes)
    if validate and p.checksums is not None:
        for i in range(nb):
            s = int(p.offsets[i])
            if p.checksums[i] != 0 and xxh3_64(p.data[s: s + int(p.sizes[i])].tobytes()) != p.checksums[i]:
                raise ValueError(f"block {i} checksum mismatch")
    d = np.zeros(nb, dtype=BLOCK_DESC)
    d["src_off"] = p.offsets
    d["src_len"] = p.sizes
    bs = p.header.block_size
    d["dst_off"] = np.arange(nb, dtype=np.uint64) * bs
    exp = np.full(nb, bs, dtype=np.uint32)
    if nb:
        exp[-1] = p.expected_size(nb - 1)
    d["dst_cap"] = exp
    d["out_size"] = exp
    out, st = lz4_decompress_batch(p.data, d, p.header.original_size, threads)
    bad = np.nonzero(st["code"])[0]
    if len(bad):
        raise ValueError(f"block {bad[0]} failed with code {st['code'][bad[0]]}")
    short = np.nonzero(st["written"] != exp)[0]
    if len(short):
        # the reference truncates the block and concatenates (decompress.rs:63-68)
        parts = [out[i * bs: i * bs + int(st["written"][i])] for i in range(nb)]
        return np.concatenate(parts)
    return out


def tensor_dims(shape) -> tuple[int, int]:
    """(rows, cols) of the 2-D transform: rank-1 tensors are one row."""
    shape = [int(s) for s in shape]
    if len(shape) == 1:
        return 1, shape[0]
    rows = int(np.prod(shape[:-1]))
    return rows, shape[-1]


def encode_spectral_q4(w: np.ndarray, retention: float = 0.30, version: int = 1,
                       block_size: int = DEFAULT_BLOCK_SIZE, threads: int = 0,
                       return_parts: bool = False, dct: str = "f32"):
    """Encode a tensor as an HCT-Q4 file (DCT -> top-k bitmap -> INT4 -> LZ4 HCT).

    dct: "f32" is the restatement of dct.rs:282-308 (f32 Makhoul FFT); "f64"
    takes the float64 orthonormal DCT-II (scipy) rounded once to float32, the
    correctly rounded coefficients, which any float64 DCT reproduces."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, n = tensor_dims(w.shape)
    if dct == "f64":
        from . import dct_2d_f64_truth

        coeffs = dct_2d_f64_truth(w.reshape(m, n)).astype(np.float32)
    else:
        coeffs = dct_2d(w.reshape(m, n), threads)
    total = m * n
    k = retain_count(total, retention)
    bm = topk_bitmap(coeffs, k, threads)
    vals = gather_retained(coeffs, bm)
    q = quantize_int4_np(vals)
    payload = np.concatenate([bm, q])
    f = write_hct(payload, list(w.shape), DTYPE_I4, FLAG_SPECTRAL_Q4, version, block_size,
                  threads=threads)
    if return_parts:
        return f, dict(coeffs=coeffs, bitmap=bm, values=vals, int4=q, payload=payload, k=k)
    return f


def split_spectral_payload(payload: np.ndarray, m: int, n: int):
    total = m * n
    bmb = (total + 7) // 8
    bm = payload[:bmb]
    k = popcount(bm)
    return bm, k, payload[bmb:]


def decode_spectral_q4_cpu(file: bytes, threads: int = 0, stage: str = "output"):
    """CPU decode of an HCT-Q4 file; stage in {"payload", "coeffs", "output"}."""
    p = parse_hct(file)
    payload = decompress_all_cpu(p, threads)
    if stage == "payload":
        return payload
    m, n = tensor_dims(p.header.shape)
    bm, k, q = split_spectral_payload(payload, m, n)
    vals = dequantize_int4(q, k)
    dense = scatter_retained(vals, bm, m * n).reshape(m, n)
    if stage == "coeffs":
        return dense
    return idct_2d(dense, threads)


def encode_int4_hct(w: np.ndarray, version: int = 1, block_size: int = DEFAULT_BLOCK_SIZE,
                    threads: int = 0) -> bytes:
    """INT4 + LZ4 HCT on raw weights (examples/safetensors_to_int4_hct.rs:241-284)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    q = quantize_int4_np(w.reshape(-1))
    return write_hct(q, list(w.shape), DTYPE_I4, 0, version, block_size, threads=threads)


def decode_int4_hct_cpu(file: bytes, threads: int = 0) -> np.ndarray:
    p = parse_hct(file)
    payload = decompress_all_cpu(p, threads)
    n = int(np.prod([int(s) for s in p.header.shape]))
    return dequantize_int4(payload, n)


# ------------------------------------------------------------ seeded generators

# ------------------------------------------------------------------ HCT V3 fragments
#
# The fragment container that haagenti-cuda's GpuDecompressor decodes
# (crates/haagenti-cuda/src/decompress.rs:322-438) and the reference's own C
# decoder reads (ref/c/hct_decoder.h:322-394):
#   [num_fragments u16], then per fragment
#   [index u16][flags u16][checksum u64][data_len u32][data: data_len bytes]
#   data = [num_coefficients u32][bitmap ceil(rows*cols/8)][f16 x num_coefficients]
# Fragments are applied in order: each writes its coefficients (in index
# order) at its bitmap's set bits, the rest of the matrix stays zero; then the
# 2-D IDCT of rows x cols.

def encode_hct_v3(w: np.ndarray, retention: float = 0.30, num_fragments: int = 1,
                  threads: int = 0) -> bytes:
    """Writer (tests and bench): DCT -> top-k -> f16 values, the retained set split in
    index order over ``num_fragments`` fragments with disjoint bitmaps."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, n = tensor_dims(w.shape)
    coeffs = dct_2d(w.reshape(m, n), threads).reshape(-1)
    total = m * n
    k = retain_count(total, retention)
    bm = topk_bitmap(coeffs, k, threads)
    idx = np.nonzero(np.unpackbits(bm, bitorder="little")[:total])[0]
    out = [struct.pack("<H", num_fragments)]
    for f, part in enumerate(np.array_split(idx, num_fragments)):
        fb = np.zeros((total + 7) // 8, np.uint8)
        np.bitwise_or.at(fb, part // 8, (1 << (part % 8)).astype(np.uint8))
        vals = coeffs[part].astype(np.float16)  # round to nearest even, as half::f16::from_f32
        data = struct.pack("<I", part.size) + fb.tobytes() + vals.tobytes()
        out.append(struct.pack("<HHQI", f, 0, xxh3_64(data), len(data)))
        out.append(data)
    return b"".join(out)


def parse_hct_v3(data: bytes, total: int) -> list:
    """Fragments as hct_decoder.h:330-373 accepts them: (bitmap, f16 values)."""
    frags = []
    if len(data) < 2 or total == 0:
        return frags
    nfrag = struct.unpack_from("<H", data, 0)[0]
    pos = 2
    bmb = (total + 7) // 8
    for _ in range(nfrag):
        if pos >= len(data) or pos + 16 > len(data):
            break
        dlen = struct.unpack_from("<I", data, pos + 12)[0]
        pos += 16
        if pos + dlen > len(data):
            break
        fd = data[pos:pos + dlen]
        pos += dlen
        if dlen < 4:
            continue
        ncoef = struct.unpack_from("<I", fd, 0)[0]
        if 4 + bmb > dlen or 4 + bmb + 2 * ncoef > dlen:
            continue
        frags.append((np.frombuffer(fd, np.uint8, bmb, 4),
                      np.frombuffer(fd, np.float16, ncoef, 4 + bmb)))
    return frags


def decode_hct_v3_cpu(data: bytes, rows: int, cols: int, threads: int = 0) -> np.ndarray:
    """hct_decoder.h:322-394 restated: scatter every fragment, then the oracle IDCT."""
    total = rows * cols
    dense = np.zeros(total, np.float32)
    for bm, vals in parse_hct_v3(data, total):
        pos = np.nonzero(np.unpackbits(bm, bitorder="little")[:total])[0][: vals.size]
        dense[pos] = vals[: pos.size].astype(np.float32)
    return idct_2d(dense.reshape(rows, cols), threads)


def gen_weight(shape, seed: int, outlier_frac: float = 0.01, std: float = 0.02,
               threads: int = 0) -> np.ndarray:
    """N(0, std) f32: 2^22-element chunks, chunk i from PCG64(SeedSequence(seed).spawn(n)[i]);
    the first 1% of a default_rng([seed, 1]) column permutation is scaled x10.
    Chunks are filled by ``threads`` threads (0: all cores); the result does
    not depend on the thread count."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    shape = tuple(int(s) for s in shape)
    n = int(np.prod(shape))
    chunk = 1 << 22
    nch = max(1, (n + chunk - 1) // chunk)
    w = np.empty(n, np.float32)
    seqs = np.random.SeedSequence(seed).spawn(nch)

    def fill(i):
        a, b = i * chunk, min(n, (i + 1) * chunk)
        np.random.Generator(np.random.PCG64(seqs[i])).standard_normal(out=w[a:b], dtype=np.float32)
        w[a:b] *= np.float32(std)

    workers = min(nch, threads if threads > 0 else (os.cpu_count() or 1))
    if workers <= 1:
        for i in range(nch):
            fill(i)
    else:
        with ThreadPoolExecutor(max_workers=workers) as ex:
            list(ex.map(fill, range(nch)))
    w = w.reshape(shape)
    if outlier_frac > 0 and len(shape) == 2:
        nout = max(1, int(shape[1] * outlier_frac))
        w[:, np.random.default_rng([seed, 1]).permutation(shape[1])[:nout]] *= np.float32(10.0)
    return w
