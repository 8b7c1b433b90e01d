"""HCT container (tensor.rs) and the composite spectral payload, CPU oracle side."""
import struct

import numpy as np
import pytest

from oracle import hct as OH


def test_header_roundtrip_v1_v2():
    # tensor.rs:1055+ header round trip
    h = OH.HctHeader(OH.ALGO_ZSTD, OH.DTYPE_I4, 0, 1234, 567, 16384, 3, [4096, 4096], 1)
    b = h.to_bytes()
    assert len(b) == 64 and b[:4] == b"HCTN"
    g = OH.HctHeader.from_bytes(b)
    assert (g.algorithm, g.dtype, g.original_size, g.compressed_size, g.block_size,
            g.num_blocks, g.shape) == (1, 4, 1234, 567, 16384, 3, [4096, 4096])
    h2 = OH.HctHeader(0, 4, OH.FLAG_HEADER_CHECKSUM, 10, 5, 16384, 1, [10], 2)
    b2 = h2.to_bytes()
    assert struct.unpack_from("<Q", b2, 56)[0] == OH.xxh3_64(b2[:56])


def test_bad_magic_and_version():
    b = bytearray(OH.HctHeader(shape=[1]).to_bytes())
    b[0] = ord("X")
    with pytest.raises(ValueError):
        OH.HctHeader.from_bytes(bytes(b))


@pytest.mark.parametrize("version", [1, 2])
def test_container_roundtrip(version):
    rng = np.random.default_rng(version)
    payload = rng.integers(0, 8, 50_000, dtype=np.uint8)
    f = OH.write_hct(payload, [50_000], OH.DTYPE_I8, 0, version)
    p = OH.parse_hct(f)
    assert p.header.num_blocks == 4 and p.header.original_size == 50_000
    assert [p.expected_size(i) for i in range(4)] == [16384, 16384, 16384, 50_000 - 3 * 16384]
    assert np.array_equal(OH.decompress_all_cpu(p), payload)


def test_v2_checksums_detect_corruption():
    rng = np.random.default_rng(9)
    payload = rng.integers(0, 255, 40_000, dtype=np.uint8)
    f = bytearray(OH.write_hct(payload, [40_000], OH.DTYPE_I8, 0, 2))
    p = OH.parse_hct(bytes(f))
    assert p.checksums is not None and (p.checksums != 0).all()
    f[-5] ^= 0xFF  # inside the last block
    with pytest.raises(ValueError, match="checksum"):
        OH.decompress_all_cpu(OH.parse_hct(bytes(f)))
    g = bytearray(OH.write_hct(payload, [40_000], OH.DTYPE_I8, 0, 2))
    g[40] ^= 1  # a shape byte under the header checksum
    with pytest.raises(ValueError, match="header checksum"):
        OH.parse_hct(bytes(g))


@pytest.mark.parametrize("shape", [(16, 16), (33, 47), (1, 100), (100, 1), (64, 512)])
def test_spectral_q4_roundtrip(shape):
    w = OH.gen_weight(shape, 11)
    f, parts = OH.encode_spectral_q4(w, return_parts=True)
    p = OH.parse_hct(f)
    assert p.header.flags & OH.FLAG_SPECTRAL_Q4 and p.header.dtype == OH.DTYPE_I4
    m, n = OH.tensor_dims(shape)
    assert parts["k"] == int(np.float32(m * n) * np.float32(0.30)) or parts["k"] == 1
    coeffs = OH.decode_spectral_q4_cpu(f, stage="coeffs")
    assert np.count_nonzero(parts["bitmap"]) > 0
    rec = OH.decode_spectral_q4_cpu(f)
    cos = float((rec.reshape(-1) * w.reshape(-1)).sum() /
                np.sqrt((rec ** 2).sum() * (w ** 2).sum()))
    assert cos > 0.5  # 30% retention of white noise keeps most of the energy
    assert coeffs.shape == (m, n)


def test_int4_container_roundtrip():
    w = OH.gen_weight((64, 96), 0)
    f = OH.encode_int4_hct(w)
    d = OH.decode_int4_hct_cpu(f)
    assert d.size == w.size
    assert np.all(np.abs(d - w.reshape(-1)) <= np.abs(w.reshape(-1)).max() / 7 * 0.5 + 1e-3)


def test_generator_shapes_and_outliers():
    w = OH.gen_weight((128, 200), 0)
    assert w.dtype == np.float32 and w.shape == (128, 200)
    col_std = w.std(axis=0)
    assert (col_std > 0.1).sum() == 2  # 1% of 200 columns scaled x10


# ---- HCT V3 fragment containers (decompress.rs:322-438, hct_decoder.h:322-394)

def test_v3_oracle_matches_reference_c_decoder(golden):
    """The oracle's restatement against hct_decode's own outputs (golden)."""
    from oracle import hct as OH

    for case in golden["ref_c_v3"]:
        got = OH.decode_hct_v3_cpu(bytes.fromhex(case["data"]), case["rows"], case["cols"])
        ref = np.array(case["out"], np.float32).reshape(case["rows"], case["cols"])
        assert np.abs(got - ref).max() <= 1e-5 + 1e-4 * np.abs(ref).max(), case["name"]


def test_v3_encoder_roundtrip_within_retention():
    from oracle import hct as OH

    w = OH.gen_weight((64, 96), 7)
    for nf in (1, 2, 4):
        d = OH.encode_hct_v3(w, 1.0, nf)
        assert len(OH.parse_hct_v3(d, w.size)) == nf
        back = OH.decode_hct_v3_cpu(d, 64, 96)
        assert np.abs(back - w).max() < 2e-3  # f16 coefficients, full retention
