"""HoloTensor oracle (oracle/holo.py) against the known answers of the
reference's own tests (crates/haagenti-hct/src/holotensor.rs, tests module)
and the documented byte layout; the library writer against the oracle.
CPU only."""
import struct

import numpy as np
import pytest

from oracle import holo as OHo


def test_quality_curve_known_answers():
    lin = ((0.0, 1.0, 0.0, 0.0), 1)
    # test_quality_curve_linear / _predict_edge_cases (holotensor.rs:2417-2434)
    assert OHo.curve_predict(*lin, 0, 8) == 0.0
    assert abs(OHo.curve_predict(*lin, 4, 8) - 0.5) < 0.01
    assert OHo.curve_predict(*lin, 8, 8) == 1.0
    assert OHo.curve_predict(*lin, 0, 0) == 0.0
    assert OHo.curve_predict(*lin, 10, 8) == 1.0
    # test_quality_curve_predict_respects_min_fragments
    m3 = ((0.0, 1.0, 0.0, 0.0), 3)
    assert OHo.curve_predict(*m3, 1, 8) == 0.0 and OHo.curve_predict(*m3, 2, 8) == 0.0
    assert OHo.curve_predict(*m3, 3, 8) > 0.0
    # test_quality_curve_spectral_shape: baseline above 0.5, increasing
    sp = (OHo.DEFAULT_CURVES[OHo.ENC_SPECTRAL][0], 1)
    q1, q4, q8 = (OHo.curve_predict(*sp, k, 8) for k in (1, 4, 8))
    assert q1 > 0.5 and q4 > q1 and q8 > q4
    # test_quality_curve_interpolation_smooth / _extrapolation_beyond_sufficient
    qs = [OHo.curve_predict(*lin, k, 8) for k in range(9)]
    assert all(b >= a for a, b in zip(qs, qs[1:]))
    assert abs(OHo.curve_predict(*lin, 100, 8) - 1.0) < 0.01
    # spectral curve values, f32 arithmetic: 0.6 + 0.3 x + 0.08 x^2 + 0.02 x^3 at x = 1/2
    assert abs(OHo.curve_predict(*sp, 4, 8) - (0.6 + 0.15 + 0.02 + 0.0025)) < 1e-6


def test_header_layout_and_roundtrip():
    # test_header_serialization_roundtrip (holotensor.rs:2596-2619)
    h = OHo.HoloHeader(OHo.ENC_LRDF, OHo.ALGO_ZSTD, 0x0003, 16, 1, 2048 * 2048 * 2, 0xDEADBEEF,
                       2, [2048, 2048], OHo.DEFAULT_CURVES[OHo.ENC_LRDF][0])
    b = OHo.header_to_bytes(h)
    assert len(b) == 96
    # offsets of the documented layout (holotensor.rs:381-403)
    assert b[0:4] == b"HTNS" and struct.unpack_from("<I", b, 4)[0] == 1
    assert b[8] == 2 and b[9] == 1 and struct.unpack_from("<HHH", b, 10) == (3, 16, 1)
    assert struct.unpack_from("<QQ", b, 16) == (2048 * 2048 * 2, 0xDEADBEEF)
    assert b[32] == 2 and b[33] == 2
    assert struct.unpack_from("<4Q", b, 34) == (2048, 2048, 0, 0)
    assert b[82:88] == bytes(6)
    r = OHo.header_from_bytes(b)
    assert (r.encoding, r.compression, r.total_fragments, r.seed, r.dtype, r.shape) == \
        (2, 1, 16, 0xDEADBEEF, 2, [2048, 2048])
    # test_header_invalid_magic / test_header_checksum_validation
    with pytest.raises(OHo.HoloError):
        OHo.header_from_bytes(b"XXXX" + b[4:])
    bad = bytearray(b)
    bad[20] ^= 1
    with pytest.raises(OHo.HoloError, match="checksum"):
        OHo.header_from_bytes(bytes(bad))


def test_writer_size_and_sv03_layout():
    # test_writer_calculates_correct_size (holotensor.rs:3171-3192)
    data = np.arange(16, dtype=np.float32).reshape(4, 4)
    f = OHo.encode_spectral(data, num_fragments=2)
    p = OHo.parse_holotensor(f)
    frag_bytes = sum(e[3] for e in p.entries)
    assert len(f) == 96 + 2 * 24 + frag_bytes
    # SpectralEncoder::encode_2d (holotensor.rs:754-776): 20-byte header + 4 B per value
    idx, body = OHo.read_fragment(p, 1)
    assert idx == 1 and len(body) == 20 + 4 * 8
    assert struct.unpack_from("<5I", body, 0) == (0x33305653, 16, 2, 1, 8)


def test_spectral_reconstruction_known_answers():
    # test_spectral_encode_decode_full (holotensor.rs:2797-2826): MSE < 0.1
    data = np.sin(np.arange(64, dtype=np.float32) * np.float32(0.1)).reshape(8, 8)
    f = OHo.encode_spectral(data, num_fragments=4)
    x, q = OHo.decode_cpu(f)
    assert float(((x - data) ** 2).mean()) < 0.1 and q == 1.0
    # test_spectral_partial_reconstruction / _quality_improves (:2829-2863)
    ramp = np.arange(64, dtype=np.float32).reshape(8, 8)
    f8 = OHo.encode_spectral(ramp, num_fragments=8)
    qs = [OHo.decode_cpu(f8, k)[1] for k in range(1, 9)]
    assert qs[1] > 0.0 and all(b >= a for a, b in zip(qs, qs[1:]))
    assert qs == [k / 8 for k in range(1, 9)]


def test_reader_rules():
    ramp = np.arange(64, dtype=np.float32).reshape(8, 8)
    f = OHo.encode_spectral(ramp, num_fragments=8)
    p = OHo.parse_holotensor(f)
    # test_reader_progressive_loading (:3101-3124): fragment i has index i
    assert [OHo.read_fragment(p, i)[0] for i in range(8)] == list(range(8))
    # test_read_to_quality (:3127-3151): stops once the curve reaches 0.75
    k = OHo.fragments_for_quality(p, 0.75)
    h = p.header
    assert 1 <= k <= 8 and OHo.curve_predict(h.curve, h.min_fragments, k, 8) >= 0.75
    # test_checksum_verification (:3195-3223)
    bad = bytearray(f)
    bad[96 + 8 * 24] ^= 0xFF
    with pytest.raises(OHo.HoloError, match="checksum"):
        OHo.read_fragment(OHo.parse_holotensor(bytes(bad)), 0)
    # fragment i not found
    with pytest.raises(OHo.HoloError, match="not found"):
        OHo.read_fragment(p, 8)
    # test_decode_corrupted_fragment_data (:3723-3739): a 4-byte fragment is an error
    dec = OHo.SpectralDecoderCpu(8, 8)
    with pytest.raises(OHo.HoloError, match="too short"):
        dec.add_fragment(bytes(4))


def test_shapes_and_inline_form():
    # test_encode_1d_preserves_original_shape / _nd_preserves_arbitrary_shape (:3885-3967)
    v = np.linspace(-1, 1, 576, dtype=np.float32)
    p1 = OHo.parse_holotensor(OHo.encode_spectral(v, num_fragments=3))
    assert p1.header.shape == [576] and OHo.matrix_dims(p1.header.shape) == (1, 576)
    t = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    p3 = OHo.parse_holotensor(OHo.encode_spectral(t, num_fragments=4))
    assert p3.header.shape == [2, 3, 4] and OHo.matrix_dims(p3.header.shape) == (2, 12)
    x, _ = OHo.decode_cpu(OHo.encode_spectral(t, num_fragments=4))
    assert np.abs(x - t.reshape(2, 12)).max() < 1e-4
    # inline form (holotensor.rs:1978-2003): total_fragments = 0, one entry after the header
    w = np.arange(16, dtype=np.float32).reshape(4, 4)
    body = OHo.sv03_fragments(OHo.dct_2d(w), 1)[0]
    h = OHo.HoloHeader(total_fragments=0, shape=[4, 4], original_size=64)
    f = OHo.header_to_bytes(h) + OHo.index_entry_bytes(0, 0, 0, len(body), len(body),
                                                       OHo.xxh3_64(body)) + body
    p = OHo.parse_holotensor(f)
    assert p.inline and OHo.total_fragments(p) == 1
    x, q = OHo.decode_cpu(f)
    assert q == 1.0 and np.abs(x - w).max() < 1e-4


def test_library_writer_matches_oracle():
    from haagenti_b200 import encode as E

    for shape, nf in (((16, 24), 5), ((576,), 3), ((2, 3, 4), 4), ((7, 9), 1)):
        w = np.random.default_rng(sum(shape)).standard_normal(shape).astype(np.float32)
        rows, cols = OHo.matrix_dims(list(shape))
        c = E.dct_2d(w.reshape(rows, cols))
        assert E.encode_holotensor(w, nf, coeffs=c) == OHo.encode_spectral(w, num_fragments=nf,
                                                                          coeffs=c)
