"""Zstandard: the libzstd oracle (oracle/zstd_ref.py) and the host-side frame
header parse of the library (hct_b200_zstd_content_size).  CPU only."""
import struct

import numpy as np
import pytest


def _data(kind, n, seed=0):
    rng = np.random.default_rng(seed)
    if kind == "random":
        return rng.integers(0, 256, n, dtype=np.uint8).tobytes()
    if kind == "zeros":
        return bytes(n)
    if kind == "fp16":
        return (rng.standard_normal(n // 2) * 0.02).astype(np.float16).tobytes()
    words = [b"alpha ", b"beta ", b"gamma ", b"tensor ", b"weight ", b"block "]
    out = b"".join(words[i] for i in rng.integers(0, len(words), n // 4 + 1))
    return out[:n]


def test_oracle_roundtrip():
    from oracle import zstd_ref as Z

    assert Z.version() >= 10400
    for kind in ("random", "zeros", "fp16", "text"):
        for n in (0, 1, 1000, 200_000):
            d = _data(kind, n, n)
            for lv in (1, 3, 19):
                c = Z.compress(d, lv, checksum=True)
                ok, out = Z.decompress(c, n + 16)
                assert ok and out == d


def test_content_size_parse():
    import haagenti_b200 as H
    from oracle import zstd_ref as Z

    d1, d2 = _data("text", 50_000, 1), _data("fp16", 70_000, 2)
    c1 = Z.compress(d1, 3)
    c2 = Z.compress(d2, 5, checksum=True)
    skip = struct.pack("<II", 0x184D2A53, 4) + b"abcd"
    assert H.ZstdDecompressor.content_size(c1) == len(d1)
    assert H.ZstdDecompressor.content_size(c1 + skip + c2) == len(d1) + len(d2)
    assert H.ZstdDecompressor.content_size(Z.compress(d1, 3, content_size=False)) is None
    assert H.ZstdDecompressor.content_size(b"") == 0
    with pytest.raises(H.CorruptedData):
        H.ZstdDecompressor.content_size(c1[:-3])
    with pytest.raises(H.CorruptedData):
        H.ZstdDecompressor.content_size(b"\x00\x01\x02\x03\x04\x05")
