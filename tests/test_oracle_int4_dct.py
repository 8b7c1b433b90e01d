"""Pins the INT4 and DCT oracles to the reference's tests, its specification
vectors and its own C decoder's outputs.  CPU only."""
import numpy as np
import pytest


# ------------------------------------------------------------- INT4

def test_int4_compressed_size_kats(orc):
    # quantization.rs:291-300
    assert orc.int4_compressed_size(32) == 18
    assert orc.int4_compressed_size(64) == 36
    assert orc.int4_compressed_size(33) == 21
    assert orc.int4_compressed_size(0) == 0


def test_int4_roundtrip_bound(orc):
    # quantization.rs:229-249
    w = ((np.arange(100) - 50) / 10).astype(np.float32)
    d = orc.dequantize_int4(orc.quantize_int4(w), 100)
    assert d.shape == (100,)
    assert np.all(np.abs(w - d) < np.abs(w) * 0.15 + 0.1)


def test_int4_sign_zero_empty(orc):
    # quantization.rs:251-270, 335-355
    assert orc.quantize_int4(np.zeros(0, np.float32)) == b""
    assert orc.dequantize_int4(b"", 0).size == 0
    assert len(orc.quantize_int4(np.ones(32, np.float32))) == 2 + 16
    d = orc.dequantize_int4(orc.quantize_int4(np.array([-5.0, 5.0, -2.5, 2.5], np.float32)), 4)
    assert d[0] < 0 < d[1] and d[2] < 0 < d[3]
    z = orc.dequantize_int4(orc.quantize_int4(np.zeros(64, np.float32)), 64)
    assert np.all(np.abs(z) < 1e-6)


def test_f16_conversions(orc):
    # quantization.rs:272-288 tolerance test
    for v in [0.0, 1.0, -1.0, 0.5, 100.0, -100.0, 0.001]:
        r = orc.f16_bits_to_f32(orc.f32_to_f16_bits(v))
        assert abs(v - r) < abs(v) * 0.01 + 0.001
    # f16 -> f32 is exact for every finite f16 (compare with numpy)
    bits = np.arange(0, 1 << 16, dtype=np.uint16)
    ours = np.array([orc.f16_bits_to_f32(int(b)) for b in bits[::97]], np.float32)
    ref = bits[::97].view(np.float16).astype(np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(ours[fin], ref[fin])
    # f32 -> f16 truncates the mantissa and flushes subnormals (quantization.rs:136-163)
    assert orc.f32_to_f16_bits(1.0 + 2 ** -11) == 0x3C00  # would round up under RNE? no: tie
    assert orc.f32_to_f16_bits(1.0 + 3 * 2 ** -12) == 0x3C00  # RNE gives 0x3C01
    assert orc.f32_to_f16_bits(1e-6) == 0x0000  # subnormal in f16 -> 0
    assert orc.f32_to_f16_bits(70000.0) == 0x7C00  # overflow -> inf


def _numpy_dequant(data: bytes, n: int) -> np.ndarray:
    """Independent numpy statement of quantization.rs:82-131."""
    if n == 0:
        return np.zeros(0, np.float32)
    nb = (n + 31) // 32
    buf = np.frombuffer(data, np.uint8)
    if len(buf) < 2 * nb:
        return np.zeros(0, np.float32)
    scales = buf[: 2 * nb].view("<f2").astype(np.float32)
    packed = buf[2 * nb:]
    m = min(n, 2 * len(packed))
    nib = np.empty(2 * len(packed), np.uint8)
    nib[0::2] = packed & 0xF
    nib[1::2] = packed >> 4
    q = nib[:m].astype(np.int8) - 8
    return (q.astype(np.float32) * scales[np.arange(m) // 32]).astype(np.float32)


def test_int4_dequant_matches_numpy_statement(orc):
    rng = np.random.default_rng(0)
    for n in [1, 2, 31, 32, 33, 63, 64, 65, 1000, 4097]:
        w = (rng.standard_normal(n) * 0.02).astype(np.float32)
        w[rng.integers(0, n)] *= 10
        q = orc.quantize_int4(w)
        assert len(q) == orc.int4_compressed_size(n)
        a = orc.dequantize_int4(q, n)
        b = _numpy_dequant(q, n)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        # short inputs: scales missing -> empty; nibbles short -> truncated
        assert orc.dequantize_int4(q[: 2 * ((n + 31) // 32) - 1], n).size == 0
        cut = q[: len(q) - 1]
        assert orc.dequantize_int4(cut, n).size == min(n, 2 * (len(cut) - 2 * ((n + 31) // 32)))


def test_quantize_rounding_rules(orc):
    # scale = max|x|/7 (f32), q = round-half-away(x/scale) clamped to [-8, 7]
    w = np.array([7.0, 3.5, -3.5, 0.5, -0.5, 2.5, -7.0] + [0.0] * 25, np.float32)
    q = np.frombuffer(orc.quantize_int4(w), np.uint8)
    nib = np.empty(32, np.int32)
    nib[0::2] = q[2:] & 0xF
    nib[1::2] = q[2:] >> 4
    assert list(nib[:7] - 8) == [7, 4, -4, 1, -1, 3, -7]


# ------------------------------------------------------------- DCT

def test_spec_vector_b1(orc, golden):
    v = golden["spec_dct"]
    x = np.array(v["input"], np.float32).reshape(v["shape"])
    c = orc.dct_2d(x).reshape(-1)
    np.testing.assert_allclose(c, np.array(v["dct_coefficients"], np.float32), atol=1e-5)
    # retained indices = top-k by |c| with ties to the lower index
    k = orc.retain_count(16, v["retention"])
    bm = orc.topk_bitmap(c, k)
    sel = [i for i in range(16) if bm[i // 8] >> (i % 8) & 1]
    assert sorted(v["retained_indices"][:k]) == sel
    rec = orc.idct_2d(orc.scatter_retained(orc.gather_retained(c, bm), bm, 16).reshape(4, 4))
    cos = float((rec * x).sum() / np.sqrt((rec * rec).sum() * (x * x).sum()))
    assert abs(cos - v["expected_cosine_similarity"]) <= v["tolerance"]


def test_constant_dc(orc):
    # ref/c/test_decoder.c:170-206 and spec 7.3: DC of 4x4 of 42 is 168
    c = orc.dct_2d(np.full((4, 4), 42.0, np.float32))
    assert abs(c[0, 0] - 168.0) < 0.01
    assert np.abs(c.reshape(-1)[1:]).max() < 1e-4


@pytest.mark.parametrize("shape", [(4, 4), (8, 8), (1, 64), (64, 1), (33, 47), (7, 100),
                                   (128, 96), (35, 167), (5, 125)])
def test_idct_makhoul_vs_f64_truth(orc, shape):
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal(shape).astype(np.float32)
    t = orc.idct_2d_f64_truth(x)
    np.testing.assert_allclose(orc.idct_2d(x), t, atol=2e-5 * max(1.0, np.abs(t).max()))
    np.testing.assert_allclose(orc.dct_2d(x), orc.dct_2d_f64_truth(x), atol=2e-5 * max(1.0, np.abs(x).max() * 4))


@pytest.mark.parametrize("n", [33, 100, 1024, 4096, 8192, 14336, 28672, 32000])
def test_idct_1d_lengths_of_the_configs(orc, n):
    import scipy.fft

    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    t = scipy.fft.idct(x.astype(np.float64), type=2, norm="ortho")
    assert np.abs(orc.idct_1d(x) - t).max() < 5e-6 * np.sqrt(np.log2(n))
    assert np.abs(orc.idct_1d(orc.dct_1d(x)) - x).max() < 2e-5  # dct.rs:462-474 style


def test_reference_c_decoder_outputs(orc, golden):
    # outputs of ref/c/hct_decoder.h (compiled from the reference) on seeded inputs
    for case in golden["ref_c_idct"]:
        x = np.array(case["input"], np.float32).reshape(case["rows"], case["cols"])
        ref_idct = np.array(case["idct"], np.float32).reshape(x.shape)
        ref_dct = np.array(case["dct"], np.float32).reshape(x.shape)
        np.testing.assert_allclose(orc.idct_2d(x), ref_idct, atol=2e-5)
        np.testing.assert_allclose(orc.dct_2d(x), ref_dct, atol=2e-5)


def test_reference_test_vector_generators(orc):
    # hct_test_vectors.rs:215-285: deterministic inputs, cosine expectations of spec 7.4/7.5
    i = np.arange(64, dtype=np.float32)
    g = (np.sin(i * np.float32(0.1)) * np.cos(i * np.float32(0.073)) * np.float32(0.5)).astype(np.float32).reshape(8, 8)
    u = np.array([1.0, 0.5, 0.25, 0.125, 0.0625, 0.03125, 0.015625, 0.0078125], np.float32)
    v = u * np.array([1, -1, 1, -1, 1, -1, 1, -1], np.float32)
    lr = np.outer(u, v).astype(np.float32)
    for x, ret, floor in [(g, 0.7, 0.9999), (lr, 0.3, 0.90)]:
        c = orc.dct_2d(x).reshape(-1)
        k = max(int(np.floor(np.float32(64) * np.float32(ret))), 1)
        bm = orc.topk_bitmap(c, k)
        rec = orc.idct_2d(orc.scatter_retained(orc.gather_retained(c, bm), bm, 64).reshape(8, 8))
        cos = float((rec * x).sum() / np.sqrt((rec * rec).sum() * (x * x).sum()))
        assert cos >= floor


def test_topk_tie_break_and_count(orc):
    # compressive.rs:144-152: stable sort by |c| desc, k = (n as f32 * r) as usize, >= 1
    assert orc.retain_count(16, 0.3) == 4
    assert orc.retain_count(3, 0.1) == 1
    assert orc.retain_count(8192 * 8192, 0.30) == int(np.float32(8192 * 8192) * np.float32(0.30))
    c = np.array([1, -3, 3, 2, -3, 0, 3, 1], np.float32)
    bm = orc.topk_bitmap(c, 3)
    assert [i for i in range(8) if bm[0] >> i & 1] == [1, 2, 4]
    rng = np.random.default_rng(5)
    c = rng.standard_normal(10000).astype(np.float32)
    c[::7] = 0.5  # many ties
    for k in [1, 10, 1429, 5000, 9999, 10000]:
        bm = orc.topk_bitmap(c, k)
        order = sorted(range(len(c)), key=lambda j: (-abs(c[j]), j))[:k]
        got = np.nonzero(np.unpackbits(bm, bitorder="little")[: len(c)])[0]
        assert list(got) == sorted(order)


# ---- mixed_precision.rs:448-539 (the private INT4 pair)

def test_f16_rne_matches_ieee(orc):
    """The RNE f32 -> f16 of half::f16::from_f32, against numpy's IEEE cast."""
    rng = np.random.default_rng(7)
    mags = np.float32(10.0) ** rng.integers(-9, 6, 100000).astype(np.float32)
    vals = np.concatenate([rng.standard_normal(100000).astype(np.float32) * mags, np.array(
        [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e6, -1e6, np.inf, -np.inf, 2.0 ** -24,
         2.0 ** -25, 3 * 2.0 ** -26, 2.0 ** -14, 5.960464477539063e-08 * 1.5], np.float32)])
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    got = np.array([orc.f32_to_f16_rne(v) for v in vals], np.uint16)
    assert np.array_equal(got, ref)


def test_int4_mp_scales_and_values(orc):
    rng = np.random.default_rng(8)
    w = (rng.standard_normal(1000) * 0.02).astype(np.float32)
    q = np.frombuffer(orc.quantize_int4_mp(w), np.uint8)
    nb = (w.size + 31) // 32
    scales = q[: 2 * nb].view(np.uint16)
    for b in range(nb):
        blk = w[32 * b: 32 * b + 32]
        m = np.max(np.abs(blk))
        s = np.float32(m) / np.float32(7.0) if m > 1e-10 else np.float32(1.0)
        assert scales[b] == np.array([s], np.float32).astype(np.float16).view(np.uint16)[0]
    # nibbles equal the testing quantizer's (same f32 scale); only the stored scale differs
    q_t = np.frombuffer(orc.quantize_int4(w), np.uint8)
    assert np.array_equal(q[2 * nb:], q_t[2 * nb:])
    d = orc.dequantize_int4_mp(q.tobytes(), w.size)
    s32 = scales.view(np.float16).astype(np.float32)
    nib = np.stack([q[2 * nb:] & 15, q[2 * nb:] >> 4], 1).reshape(-1)[: w.size].astype(np.int32)
    assert np.array_equal(d, (nib - 8).astype(np.float32) * np.repeat(s32, 32)[: w.size])


def test_int4_mp_short_data_zero_fills(orc):
    w = np.linspace(-1, 1, 100, dtype=np.float32)
    q = orc.quantize_int4_mp(w)
    assert orc.dequantize_int4_mp(q, 0).size == 0
    assert orc.dequantize_int4_mp(b"", 100).size == 0
    assert np.array_equal(orc.dequantize_int4_mp(q[:5], 100), np.zeros(100, np.float32))  # < scales
    full = orc.dequantize_int4_mp(q, 100)
    cut = orc.dequantize_int4_mp(q[: 8 + 20], 100)  # 8 scale bytes + 20 nibble bytes = 40 values
    assert np.array_equal(cut[:40], full[:40]) and not cut[40:].any()
