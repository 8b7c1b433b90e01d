"""The library's writer side (encode.py + the compress_block port in the .so)
produces exactly what the oracle's restatement of the reference produces.  CPU only."""
import numpy as np
import pytest

from haagenti_b200 import encode as E


def test_quantize_int4_matches_oracle(orc):
    rng = np.random.default_rng(0)
    for n in [1, 2, 31, 32, 33, 1000, 4097, 100_001]:
        w = (rng.standard_normal(n) * rng.choice([1e-12, 0.02, 3.0, 1e5])).astype(np.float32)
        w[rng.integers(0, n, 3)] *= 10
        # exact .5 ratios exercise round-half-away-from-zero
        if n >= 32:
            w[:32] = np.float32(0.0)
            w[0], w[1], w[2] = 7.0, 3.5, -0.5
        assert np.array_equal(E.quantize_int4(w), orc.quantize_int4_np(w)), n
    assert E.quantize_int4(np.zeros(0, np.float32)).size == 0


def test_f16_truncation_matches_oracle(orc):
    vals = np.array([0.0, -0.0, 1.0, 1.0 + 3 * 2 ** -12, 1e-6, 6.1e-5, 65504.0, 70000.0,
                     np.inf, -np.inf, 0.33333334, 1e-10, 2.0 ** -14, 2.0 ** -15], np.float32)
    got = E._f32_to_f16_trunc(vals)
    ref = np.array([orc.f32_to_f16_bits(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, ref)


def test_lz4_compressor_matches_oracle(orc):
    rng = np.random.default_rng(4)
    for n in [0, 5, 12, 13, 100, 16384, 70000]:
        for kind in range(3):
            if kind == 0:
                d = rng.integers(0, 256, n, dtype=np.uint8)
            elif kind == 1:
                d = rng.integers(0, 4, n, dtype=np.uint8)
            else:
                d = np.resize(np.frombuffer(b"The quick brown fox ", np.uint8), n)
            packed, lens = E.lz4_compress_chunks(d, 16384)
            ref, rlens = orc.lz4_compress_chunks(d, 16384)
            assert np.array_equal(lens, rlens) and np.array_equal(packed, ref), (n, kind)


def test_spectral_select_matches_oracle_topk(orc):
    rng = np.random.default_rng(8)
    c = rng.standard_normal(50_000).astype(np.float32)
    c[::13] = np.float32(0.25)  # ties
    for r in [0.001, 0.3, 0.9, 1.0]:
        bm, vals = E.spectral_select(c, r)
        k = orc.retain_count(c.size, r)
        assert np.array_equal(bm, orc.topk_bitmap(c, k))
        assert np.array_equal(vals, orc.gather_retained(c, bm))


def test_written_files_decode_with_oracle(orc):
    from oracle import hct as OH

    w = E.synthetic_weight((48, 80), 3)
    assert np.array_equal(w, OH.gen_weight((48, 80), 3))
    for v in (1, 2):
        f = E.encode_spectral_q4(w, version=v)
        p = OH.parse_hct(f)
        assert p.header.flags & OH.FLAG_SPECTRAL_Q4 and p.header.version == v
        rec = OH.decode_spectral_q4_cpu(f)
        cos = float((rec * w).sum() / np.sqrt((rec * rec).sum() * (w * w).sum()))
        assert cos > 0.5
        f4 = E.encode_int4(w, version=v)
        assert np.array_equal(OH.decode_int4_hct_cpu(f4), orc.dequantize_int4(orc.quantize_int4(w), w.size))
    # same DCT as the oracle within f32 accuracy
    np.testing.assert_allclose(E.dct_2d(w), orc.dct_2d(w), atol=1e-5)


def test_quantize_int4_mp_matches_oracle(orc):
    from haagenti_b200 import encode as E

    rng = np.random.default_rng(9)
    for n in (1, 31, 32, 33, 1000, 65537):
        w = (rng.standard_normal(n) * 10.0 ** rng.integers(-8, 3)).astype(np.float32)
        w[::17] = 0.0
        assert E.quantize_int4_mp(w).tobytes() == orc.quantize_int4_mp(w), n


def test_hct_v3_writer_matches_oracle(orc):
    from haagenti_b200 import encode as E
    from oracle import hct as OH

    w = OH.gen_weight((96, 160), 12)
    c = OH.dct_2d(w)  # the same coefficients (the writers' DCTs differ in the last ulp)
    for nf in (1, 3):
        assert E.encode_hct_v3(w, 0.3, nf, coeffs=c) == OH.encode_hct_v3(w, 0.3, nf)
