"""Generates tests/golden/golden.json, the fixtures that pin the CPU oracle.

Run in the build container (it reads the reference checkout and the system
liblz4); the JSON it writes is committed so that the tests need neither.

    python tests/golden/make_golden.py [--reference /path/to/haagenti]

Contents
  lz4_roundtrip   inputs of crates/haagenti-lz4/src/block.rs:379-450 tests
  lz4_interop     standard LZ4 blocks made by liblz4 (LZ4_compress_default)
                  for the interop tests at block.rs:452-502 (the reference
                  uses lz4_flex, which emits the same block format)
  lz4_errors      corrupt / truncated blocks with the error variant and
                  position derived by hand from block.rs:261-366
  spec_dct        Appendix B.1 of docs/HCT-SPECIFICATION-DRAFT.md
  ref_c_idct      outputs of the reference's own C decoder
                  (ref/c/hct_decoder.h hct_idct_2d / hct_dct_2d, compiled into
                  oracle/_ref) on seeded inputs
  ref_c_v3        V3 fragment containers (decompress.rs:322-438 layout) and the
                  reference C decoder's hct_decode output for them: 1-3
                  fragments, a truncated trailing fragment, a fragment whose
                  coefficient count is below its bitmap's popcount
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle  # noqa: E402

LZ4_ROUNDTRIP = {
    "empty": b"",
    "small": b"Hello",
    "repetitive": b"A" * 40,
    "mixed": b"Hello, World! Hello, World! Hello, World! This is a test.",
    "large": (b"The quick brown fox jumps over the lazy dog. " * 300)[:10000],
    "interop_1": b"Hello, LZ4! This is a test for interoperability with lz4_flex.",
    "interop_2": b"Testing compression output compatibility with lz4_flex reference.",
    "interop_repetitive": (b"ABCDEFGH" * 200)[:1000],
}

# (name, block bytes, output_size, capacity, expected code, position, provided, written)
# Codes: 0 ok, 1 UnexpectedEof{bytes_read=position}, 2 BufferTooSmall{required=position,
# provided}, 3 "invalid zero offset", 4 "offset beyond output" at position.
LZ4_ERRORS = [
    # literal run longer than the input: block.rs:293-295 -> EOF at input_pos (1)
    ("literal_past_end", [0x10], 8, 8, 1, 1, 0, 0),
    # 15-literal token with no extension byte: block.rs:279-281 -> EOF(1)
    ("lit_ext_missing", [0xF0], 64, 64, 1, 1, 0, 0),
    # extension bytes of 255 that run off the end: EOF at input.len() (3)
    ("lit_ext_run_off", [0xF0, 0xFF, 0xFF], 1000, 1000, 1, 3, 0, 0),
    # zero match offset: block.rs:320-322
    ("zero_offset", [0x11, 0x61, 0x00, 0x00], 10, 10, 3, 1, 0, 1),
    # offset 2 with 1 byte of output: block.rs:323-325 -> at output_pos 1
    ("offset_beyond", [0x11, 0x61, 0x02, 0x00], 10, 10, 4, 1, 0, 1),
    # match of 5 bytes into a 3-byte buffer: block.rs:345-350 -> required 6, provided 3
    ("match_overflow", [0x11, 0x61, 0x01, 0x00], 3, 3, 2, 6, 3, 1),
    # 2 literals into a 1-byte buffer: block.rs:296-301 -> required 2, provided 1
    ("literal_overflow", [0x20, 0x61, 0x62], 1, 1, 2, 2, 1, 0),
    # match-length extension missing: block.rs:331-333 -> EOF at 4
    ("match_ext_missing", [0x1F, 0x61, 0x01, 0x00], 100, 100, 1, 4, 0, 1),
    # offset cut short: block.rs:314-316 -> EOF at 2
    ("offset_truncated", [0x10, 0x61, 0x01], 5, 5, 1, 2, 0, 1),
    # a complete block decoded with a larger expected size: no offset -> EOF(2)
    ("short_expected", [0x10, 0x61], 5, 5, 1, 2, 0, 1),
    # literals reach output_size: loop ends, trailing bytes ignored (block.rs:309)
    ("early_exit", [0x10, 0x61, 0xFF, 0xFF], 1, 1, 0, 0, 0, 1),
    # zero-length block with output_size 0
    ("empty_block", [], 0, 0, 0, 0, 0, 0),
    # token only, no literals, output_size 0 -> break
    ("token_only", [0x00], 0, 0, 0, 0, 0, 0),
    # overlapping RLE match: 'a' then offset 1 length 4+15+0=19 -> 20 bytes of 'a'
    ("rle_overlap", [0x1F, 0x61, 0x01, 0x00, 0x00], 20, 20, 0, 0, 0, 20),
    # offset 3, length 8: "abc" then "abcabcab"
    ("overlap_period3", [0x34, 0x61, 0x62, 0x63, 0x03, 0x00], 11, 11, 0, 0, 0, 11),
    # output smaller than expected size after the last sequence: Ok with fewer bytes
    ("partial_ok", [0x30, 0x61, 0x62, 0x63], 3, 10, 0, 0, 0, 3),
]


def lz4_interop(inputs):
    lz = C.CDLL("liblz4.so.1")
    lz.LZ4_compressBound.restype = C.c_int
    out = {}
    for name, data in inputs.items():
        cap = lz.LZ4_compressBound(len(data))
        dst = C.create_string_buffer(cap)
        n = lz.LZ4_compress_default(data, dst, len(data), cap)
        out[name] = dst.raw[:n].hex()
    return out


def spec_dct(reference: str):
    path = os.path.join(reference, "docs", "HCT-SPECIFICATION-DRAFT.md")
    text = open(path).read()
    block = text[text.index("### B.1 sequential_4x4"):]
    block = block[block.index("{"): block.index("}") + 1]
    return json.loads(block)


def ref_c(reference: str):
    so = os.path.join(REPO, "oracle", "_ref", "libhct_ref.so")
    if not os.path.exists(so):
        oracle.build()
    lib = C.CDLL(so)
    f32p = C.POINTER(C.c_float)
    for fn in (lib.hct_idct_2d, lib.hct_dct_2d):
        fn.restype = None
        fn.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t]
    cases = []
    for seed, (rows, cols) in enumerate([(4, 4), (8, 8), (1, 16), (16, 1), (5, 7), (16, 32),
                                         (33, 17), (64, 64)]):
        rng = np.random.default_rng(1000 + seed)
        x = (rng.standard_normal((rows, cols)) * 0.1).astype(np.float32)
        y = np.empty_like(x)
        lib.hct_idct_2d(x.ctypes.data_as(f32p), y.ctypes.data_as(f32p), rows, cols)
        z = np.empty_like(x)
        lib.hct_dct_2d(x.ctypes.data_as(f32p), z.ctypes.data_as(f32p), rows, cols)
        cases.append(dict(seed=1000 + seed, rows=rows, cols=cols,
                          input=x.reshape(-1).tolist(), idct=y.reshape(-1).tolist(),
                          dct=z.reshape(-1).tolist()))
    return cases


def ref_c_v3(reference: str):
    from oracle import hct as OH

    so = os.path.join(REPO, "oracle", "_ref", "libhct_ref.so")
    if not os.path.exists(so):
        oracle.build()
    lib = C.CDLL(so)
    lib.hct_decode.restype = C.POINTER(C.c_float)
    lib.hct_decode.argtypes = [C.c_char_p, C.c_size_t, C.c_size_t, C.c_size_t]
    libc = C.CDLL(None)
    libc.free.argtypes = [C.c_void_p]
    cases = []

    def add(name, data, rows, cols):
        p = lib.hct_decode(data, len(data), rows, cols)
        out = np.ctypeslib.as_array(p, (rows * cols,)).astype(np.float32).copy()
        libc.free(C.cast(p, C.c_void_p))
        cases.append(dict(name=name, rows=rows, cols=cols, data=data.hex(), out=out.tolist()))

    for name, (rows, cols), nf, seed in [("one_fragment", (16, 24), 1, 1),
                                         ("two_fragments", (24, 40), 2, 2),
                                         ("three_fragments_odd", (33, 17), 3, 3),
                                         ("row_vector", (1, 64), 1, 4),
                                         ("column_vector", (48, 1), 2, 5)]:
        w = OH.gen_weight((rows, cols), 2000 + seed)
        add(name, OH.encode_hct_v3(w, 0.3, nf), rows, cols)
    # the last fragment cut short: hct_decode stops before it
    w = OH.gen_weight((16, 32), 2010)
    d = OH.encode_hct_v3(w, 0.4, 2)
    add("truncated_fragment", d[:-7], 16, 32)
    # fewer coefficients than set bits: the count fields say 5 fewer
    d = bytearray(OH.encode_hct_v3(OH.gen_weight((16, 16), 2011), 0.5, 1))
    n = int.from_bytes(d[18:22], "little")
    d[18:22] = (n - 5).to_bytes(4, "little")
    d[14:18] = (int.from_bytes(d[14:18], "little") - 10).to_bytes(4, "little")
    add("short_coefficients", bytes(d[:len(d) - 10]), 16, 16)
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=oracle.reference_root(),
                    help="haagenti checkout (default: $HAAGENTI_REFERENCE or ../reference)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("no haagenti checkout found; pass --reference")
    oracle.build()
    g = {
        "generator": "tests/golden/make_golden.py",
        "lz4_roundtrip": {k: v.hex() for k, v in LZ4_ROUNDTRIP.items()},
        "lz4_interop": lz4_interop(LZ4_ROUNDTRIP),
        "lz4_errors": [dict(name=n, block=bytes(b).hex(), output_size=o, capacity=c, code=code,
                            position=p, provided=pv, written=w)
                       for (n, b, o, c, code, p, pv, w) in LZ4_ERRORS],
        "spec_dct": spec_dct(args.reference),
        "ref_c_idct": ref_c(args.reference),
        "ref_c_v3": ref_c_v3(args.reference),
    }
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(g, f, indent=1)
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    main()
