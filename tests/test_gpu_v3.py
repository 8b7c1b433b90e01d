"""HCT V3 fragment containers (bitmap + fp16 coefficients) on the GPU against
the reference's own C decoder (golden outputs of ref/c/hct_decoder.h
hct_decode) and the oracle's restatement.  Tolerance as the other IDCT
tests: max-abs <= 1e-3, cosine >= 0.99999; bf16 adds its half-ulp."""
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-3
MIN_COS = 0.99999


def _cos(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    na, nb = np.sqrt((a * a).sum()), np.sqrt((b * b).sum())
    if na == 0 or nb == 0:
        return 1.0 if na == nb else 0.0
    return float((a * b).sum() / (na * nb))


def test_v3_reference_c_decoder_vectors(hb, golden):
    for case in golden["ref_c_v3"]:
        rows, cols = case["rows"], case["cols"]
        ref = np.array(case["out"], np.float32).reshape(rows, cols)
        got = hb.hct_v3_decode(bytes.fromhex(case["data"]), rows, cols).cpu().numpy()
        err = np.abs(got.astype(np.float64) - ref).max()
        assert err <= MAX_ABS and _cos(got, ref) >= MIN_COS, (case["name"], err)


@pytest.mark.parametrize("shape,nf", [((256, 512), 1), ((1024, 8192), 3), ((300, 1000), 2),
                                      ((1, 4096), 1), ((4096, 1), 2), ((8192, 1024), 1)])
def test_v3_decode_vs_oracle(hb, shape, nf):
    from oracle import hct as OH

    w = OH.gen_weight(shape, 60 + nf)
    data = OH.encode_hct_v3(w, 0.3, nf)
    ref = OH.decode_hct_v3_cpu(data, *shape)
    dec = hb.HctV3Decoder(data, *shape)
    assert dec.num_fragments == nf
    got = dec.decode(hb.F32).cpu().numpy()
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= MAX_ABS and _cos(got, ref) >= MIN_COS, (shape, err)
    bf = dec.decode(hb.BF16).float().cpu().numpy()
    assert (np.abs(bf - ref) <= MAX_ABS + 2.0 ** -8 * np.abs(ref)).all()
    again = dec.decode(hb.F32).cpu().numpy()  # decode is repeatable
    assert np.array_equal(again, got)


def test_v3_overlapping_fragments_later_wins(hb):
    """Two fragments with the same bitmap: the second's values replace the first's."""
    from oracle import hct as OH

    shape = (64, 128)
    a = OH.encode_hct_v3(OH.gen_weight(shape, 1), 0.3, 1)
    b = OH.encode_hct_v3(OH.gen_weight(shape, 2), 0.3, 1)
    both = struct.pack("<H", 2) + a[2:] + b[2:]
    ref = OH.decode_hct_v3_cpu(both, *shape)
    got = hb.hct_v3_decode(both, *shape).cpu().numpy()
    assert np.abs(got - ref).max() <= MAX_ABS and _cos(got, ref) >= MIN_COS


def test_v3_edge_cases(hb):
    from oracle import hct as OH

    with pytest.raises(hb.CorruptedData, match="too short"):
        hb.hct_v3_decode(b"\x01", 8, 8)
    z = hb.hct_v3_decode(struct.pack("<H", 0), 16, 32).cpu().numpy()  # no fragments
    assert not z.any()
    d = OH.encode_hct_v3(OH.gen_weight((32, 64), 3), 0.5, 2)
    cut = d[: len(d) - 9]  # the second fragment runs past the end: decoded without it
    ref = OH.decode_hct_v3_cpu(cut, 32, 64)
    got = hb.hct_v3_decode(cut, 32, 64).cpu().numpy()
    assert np.abs(got - ref).max() <= MAX_ABS


def test_v3_zstd_wrapped(hb):
    """decompress.rs:296-319: data that starts with the zstd magic is decoded
    first (here on the GPU); data that does not decode is parsed as it is."""
    from oracle import hct as OH
    from oracle import zstd_ref as Z

    shape = (256, 512)
    w = OH.gen_weight(shape, 90)
    data = OH.encode_hct_v3(w, 0.3, 3)
    plain = hb.hct_v3_decode(data, *shape).cpu().numpy()
    for lv, ck in ((1, False), (9, True)):
        got = hb.hct_v3_decode(Z.compress(data, lv, checksum=ck), *shape).cpu().numpy()
        assert np.array_equal(got, plain)
    # a zstd magic in front of data that is no zstd frame: parsed raw, as the
    # reference does (here a V3 container whose first bytes read as the magic)
    fake = struct.pack("<I", 0xFD2FB528) + bytes(8)
    ref = OH.decode_hct_v3_cpu(fake, *shape)
    got = hb.hct_v3_decode(fake, *shape).cpu().numpy()
    assert np.array_equal(got, ref)
