"""Pins the LZ4 oracle (restatement of crates/haagenti-lz4/src/block.rs) to the
reference's own tests and to standard LZ4 blocks.  CPU only."""
import numpy as np
import pytest


def test_roundtrip_reference_inputs(orc, golden):
    # block.rs:379-450: empty, small, repetitive, mixed, large
    for name, hexdata in golden["lz4_roundtrip"].items():
        data = bytes.fromhex(hexdata)
        comp = orc.lz4_compress_block(data)
        assert len(comp) <= orc.max_compressed_size(len(data))
        r = orc.lz4_decompress_block(comp, len(data))
        assert r.code == 0 and r.written == len(data) and r.data == data, name
    # block.rs:408, 442: repetitive inputs shrink
    assert len(orc.lz4_compress_block(b"A" * 40)) < 40
    big = bytes.fromhex(golden["lz4_roundtrip"]["large"])
    assert len(orc.lz4_compress_block(big)) < len(big)


def test_decodes_standard_lz4_blocks(orc, golden):
    # block.rs:452-502 decode blocks produced by another LZ4 implementation
    for name, hexblock in golden["lz4_interop"].items():
        data = bytes.fromhex(golden["lz4_roundtrip"][name])
        r = orc.lz4_decompress_block(bytes.fromhex(hexblock), len(data))
        assert r.code == 0 and r.data == data, name


def test_compressed_blocks_decode_with_liblz4(orc, golden):
    # our compressor's output is standard LZ4 (block.rs:468-482)
    import ctypes as C

    try:
        lz = C.CDLL("liblz4.so.1")
    except OSError:
        pytest.skip("system liblz4 not present")
    for name, hexdata in golden["lz4_roundtrip"].items():
        data = bytes.fromhex(hexdata)
        if not data:
            continue
        comp = orc.lz4_compress_block(data)
        out = C.create_string_buffer(len(data))
        n = lz.LZ4_decompress_safe(comp, out, len(comp), len(data))
        assert n == len(data) and out.raw == data, name


def test_error_semantics(orc, golden):
    # hand-derived expectations from block.rs:261-366
    for case in golden["lz4_errors"]:
        r = orc.lz4_decompress_block(bytes.fromhex(case["block"]), case["output_size"],
                                     case["capacity"])
        assert r.code == case["code"], case["name"]
        assert r.written == case["written"], case["name"]
        if case["code"]:
            assert r.position == case["position"], case["name"]
            assert r.provided == case["provided"], case["name"]
    by = {c["name"]: c for c in golden["lz4_errors"]}
    assert orc.lz4_decompress_block(bytes.fromhex(by["rle_overlap"]["block"]), 20).data == b"a" * 20
    assert orc.lz4_decompress_block(bytes.fromhex(by["overlap_period3"]["block"]), 11).data == b"abcabcabcab"


def test_compress_small_inputs_literals_only(orc):
    # block.rs:77-79: inputs under 13 bytes are one literal run
    for n in range(13):
        data = bytes(range(n))
        comp = orc.lz4_compress_block(data)
        assert comp[0] >> 4 == min(n, 15)
        assert comp[1:] == data


def test_random_roundtrips_and_batch(orc):
    rng = np.random.default_rng(7)
    payloads = []
    for i in range(40):
        n = int(rng.integers(0, 70000))
        kind = i % 4
        if kind == 0:
            d = rng.integers(0, 256, n, dtype=np.uint8)
        elif kind == 1:
            d = rng.integers(0, 3, n, dtype=np.uint8)
        elif kind == 2:
            d = np.zeros(n, np.uint8)
        else:
            d = np.frombuffer((rng.standard_normal(n // 2 + 1) * 0.02).astype(np.float16).tobytes(),
                              np.uint8)[:n]
        payloads.append(d.tobytes())
    comps = [orc.lz4_compress_block(p) for p in payloads]
    for p, c in zip(payloads, comps):
        assert orc.lz4_decompress_block(c, len(p)).data == p
    # batch API == single-block API
    src = np.frombuffer(b"".join(comps), np.uint8)
    d = np.zeros(len(comps), dtype=orc.BLOCK_DESC)
    so, do = 0, 0
    for i, (p, c) in enumerate(zip(payloads, comps)):
        d[i] = (so, do, len(c), len(p), len(p), 0)
        so += len(c)
        do += len(p)
    out, st = orc.lz4_decompress_batch(src, d, do)
    assert (st["code"] == 0).all()
    assert out.tobytes() == b"".join(payloads)


def test_chunked_compression_matches_single_blocks(orc):
    rng = np.random.default_rng(3)
    data = rng.integers(0, 16, 100_000, dtype=np.uint8)
    packed, lens = orc.lz4_compress_chunks(data, 16384)
    assert len(lens) == 7
    pos = 0
    for i, ln in enumerate(lens):
        chunk = data[i * 16384:(i + 1) * 16384].tobytes()
        assert packed[pos:pos + ln].tobytes() == orc.lz4_compress_block(chunk)
        pos += ln
