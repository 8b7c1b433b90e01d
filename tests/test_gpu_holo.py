"""HoloTensor spectral decode on the GPU (hct_b200_holo_*) against the oracle
restatement of HoloTensorReader + SpectralDecoder (oracle/holo.py).
Tolerance as the other IDCT tests: max-abs <= 1e-3 and cosine >= 0.99999
against the oracle's f32 reconstruction (the GPU stages the coefficients and
the intermediate passes in fp16)."""
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-3
MIN_COS = 0.99999


def _cos(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float((a * b).sum() / np.sqrt((a * a).sum() * (b * b).sum()))


def _check(got, ref, tag):
    err = float(np.abs(got.astype(np.float64) - ref.astype(np.float64)).max())
    cos = _cos(got, ref)
    assert err <= MAX_ABS and cos >= MIN_COS, f"{tag}: max-abs {err:.3e} cos {cos:.8f}"


def _file(shape, nf, seed):
    from oracle import holo as OHo
    from oracle import hct as OH

    w = OH.gen_weight(shape, seed)
    return OHo.encode_spectral(w, num_fragments=nf)


@pytest.mark.parametrize("shape,nf", [((64, 96), 8), ((256, 1024), 8), ((4096,), 4),
                                      ((2, 3, 64), 3), ((8192, 1), 8), ((1024, 8192), 8),
                                      ((300, 700), 5), ((128, 2048), 1)])
def test_full_decode_vs_oracle(hb, shape, nf):
    from oracle import holo as OHo

    f = _file(shape, nf, 60 + sum(shape))
    ref, q_ref = OHo.decode_cpu(f)
    r = hb.HoloTensorReader(f)
    assert r.total_fragments == nf and r.shape == tuple(shape)
    got = r.decode().cpu().numpy()
    assert got.shape == ref.shape
    _check(got, ref, f"{shape}")
    assert r.quality == q_ref == 1.0


@pytest.mark.parametrize("k", [1, 2, 5, 7])
def test_progressive_decode(hb, k):
    from oracle import holo as OHo

    f = _file((512, 768), 8, 70)
    ref, q_ref = OHo.decode_cpu(f, k)
    r = hb.HoloTensorReader(f)
    got = r.decode(k).cpu().numpy()
    _check(got, ref, f"k={k}")
    assert r.quality == np.float32(q_ref)


def test_quality_curve_and_read_to_quality(hb):
    from oracle import holo as OHo

    f = _file((64, 64), 8, 71)
    p = OHo.parse_holotensor(f)
    r = hb.HoloTensorReader(f)
    h = p.header
    for k in range(0, 11):
        assert r.predict_quality(k) == OHo.curve_predict(h.curve, h.min_fragments, k, 8)
    for t in (0.0, 0.5, 0.75, 0.9, 0.99, 1.0, 1.5):
        assert r.fragments_for_quality(t) == OHo.fragments_for_quality(p, t)
    out, q = r.decode_to_quality(0.75)
    k = OHo.fragments_for_quality(p, 0.75)
    _check(out.cpu().numpy(), OHo.decode_cpu(f, k)[0], "to quality")
    assert q == OHo.curve_predict(h.curve, h.min_fragments, k, 8)


def test_half_outputs(hb):
    import torch
    from oracle import holo as OHo

    f = _file((256, 512), 4, 72)
    ref = torch.from_numpy(OHo.decode_cpu(f)[0])
    r = hb.HoloTensorReader(f)
    for dt, tol in ((hb.F16, 2.0 ** -11), (hb.BF16, 2.0 ** -8)):
        got = r.decode(out_dtype=dt).float().cpu()
        err = (got - ref).abs()
        assert bool((err <= MAX_ABS + tol * ref.abs()).all()), float(err.max())


def _rewrite(f, entries=None, fragments=None, header=None):
    """Rebuild a file from (possibly edited) header, index entries and bodies."""
    from oracle import holo as OHo

    p = OHo.parse_holotensor(f)
    h = header or p.header
    ents = entries if entries is not None else list(p.entries)
    bodies = fragments if fragments is not None else [
        f[p.data_offset + e[2]: p.data_offset + e[2] + e[3]] for e in p.entries]
    out = bytearray(OHo.header_to_bytes(h))
    off = 0
    for e, b in zip(ents, bodies):
        out += OHo.index_entry_bytes(e[0], e[1], off, len(b), len(b), OHo.xxh3_64(b))
        off += len(b)
    for b in bodies:
        out += b
    return bytes(out)


def test_index_order_and_overlapping_fragments(hb):
    """Fragments found by index value, not table order; fragments that do not
    partition the positions (different strides, repeated positions) follow
    the decoder's later-over-earlier rule (per-fragment scatter path)."""
    from oracle import holo as OHo

    f = _file((96, 128), 4, 73)
    p = OHo.parse_holotensor(f)
    bodies = [f[p.data_offset + e[2]: p.data_offset + e[2] + e[3]] for e in p.entries]
    rev = _rewrite(f, entries=list(reversed(p.entries)), fragments=list(reversed(bodies)))
    r = hb.HoloTensorReader(rev)
    _check(r.decode().cpu().numpy(), OHo.decode_cpu(rev)[0], "reversed table")
    # fragment 1 rewritten with stride 2 over the same coefficients: overlaps fragment 0..3
    n = 96 * 128
    dense = np.zeros(n, np.float32)
    for i, b in enumerate(bodies):
        dense[i::4] = np.frombuffer(b, np.float32, offset=20)
    odd = struct.pack("<5I", 0x33305653, n, 2, 1, n // 2) + (dense[1::2] * 0.5).tobytes()
    zero_stride = struct.pack("<5I", 0x33305653, n, 0, 5, 3) + np.array(
        [1.0, 2.0, 0.25], np.float32).tobytes()
    mixed = _rewrite(f, fragments=[bodies[0], odd, bodies[2], zero_stride])
    ref, q = OHo.decode_cpu(mixed)
    r = hb.HoloTensorReader(mixed)
    _check(r.decode().cpu().numpy(), ref, "overlapping")
    assert r.quality == np.float32(q)


def test_inline_form(hb):
    from oracle import holo as OHo
    from oracle import hct as OH

    w = OH.gen_weight((32, 256), 74)
    body = OHo.sv03_fragments(OHo.dct_2d(w), 1)[0]
    h = OHo.HoloHeader(total_fragments=0, shape=[32, 256], original_size=w.size * 4)
    f = OHo.header_to_bytes(h) + OHo.index_entry_bytes(0, 0, 0, len(body), len(body),
                                                       OHo.xxh3_64(body)) + body
    r = hb.HoloTensorReader(f)
    assert r.is_inline_format and r.total_fragments == 1
    _check(r.decode().cpu().numpy(), OHo.decode_cpu(f)[0], "inline")
    with pytest.raises(hb.CorruptedData, match="inline"):
        r.decode(2)


def test_errors(hb):
    from oracle import holo as OHo

    f = _file((64, 64), 4, 75)
    p = OHo.parse_holotensor(f)
    # header: magic, version, checksum, codes
    with pytest.raises(hb.CorruptedData):
        hb.HoloTensorReader(b"XXXX" + f[4:])
    with pytest.raises(hb.CorruptedData):
        hb.HoloTensorReader(f[:95])
    bad = bytearray(f)
    bad[20] ^= 1
    with pytest.raises(hb.ChecksumMismatch):
        hb.HoloTensorReader(bytes(bad))
    # a corrupted fragment fails only when it is read
    bad = bytearray(f)
    bad[p.data_offset + p.entries[2][2] + 30] ^= 0xFF
    r = hb.HoloTensorReader(bytes(bad))
    r.decode(2)
    with pytest.raises(hb.ChecksumMismatch):
        r.decode(3)
    r = hb.HoloTensorReader(f)
    with pytest.raises(hb.CorruptedData, match="not found"):
        r.decode(5)
    with pytest.raises(hb.CorruptedData, match="no fragments"):
        r.decode(0)
    # a fragment flagged as zstd that holds no zstd frame fails to decompress
    # (read_fragment, holotensor.rs:2081-2091); other encodings and the legacy
    # layouts are not decoded
    ents = [list(e) for e in p.entries]
    ents[1][1] = 1
    with pytest.raises(hb.CorruptedData, match="decompress"):
        hb.HoloTensorReader(_rewrite(f, entries=ents)).decode()
    h = OHo.header_from_bytes(f[:96])
    h.encoding = OHo.ENC_LRDF
    with pytest.raises(hb.Unsupported):
        hb.HoloTensorReader(_rewrite(f, header=h)).decode()
    bodies = [f[p.data_offset + e[2]: p.data_offset + e[2] + e[3]] for e in p.entries]
    short = _rewrite(f, fragments=[bodies[0], b"\x53\x56\x30\x33" + bytes(8)] + bodies[2:])
    with pytest.raises(hb.CorruptedData, match="V3 fragment too short"):
        hb.HoloTensorReader(short).decode()
    legacy = _rewrite(f, fragments=[bodies[0], struct.pack("<II", 1, 0) + bytes(8)] + bodies[2:])
    with pytest.raises(hb.Unsupported):
        hb.HoloTensorReader(legacy).decode()
    # fragments beyond the bad one are never read
    hb.HoloTensorReader(legacy).decode(1)


def test_zstd_compressed_fragments(hb):
    """Fragments stored as zstd frames (index entry flag bit 0) decode like the
    uncompressed file; a fragment whose frames do not decode fails the decode
    that reads it."""
    from oracle import holo as OHo
    from oracle import zstd_ref as Z

    f = _file((384, 1024), 6, 76)
    p = OHo.parse_holotensor(f)
    bodies = [f[p.data_offset + e[2]: p.data_offset + e[2] + e[3]] for e in p.entries]
    packed = [(i, 1, Z.compress(b, 3 + i % 3, checksum=bool(i % 2),
                               content_size=bool(i % 3))) for i, b in enumerate(bodies)]
    zf = OHo.write_holotensor(p.header, packed)
    ref, q = OHo.decode_cpu(zf)
    r = hb.HoloTensorReader(zf)
    _check(r.decode().cpu().numpy(), ref, "zstd fragments")
    assert r.quality == q == 1.0
    _check(r.decode(3).cpu().numpy(), OHo.decode_cpu(zf, 3)[0], "zstd fragments, k=3")
    bad = list(packed)
    frame = bytearray(bad[4][2])
    frame[len(frame) // 2] ^= 0xFF
    frame[-5] ^= 0x5A
    bad[4] = (4, 1, bytes(frame))
    bf = OHo.write_holotensor(p.header, bad)
    r = hb.HoloTensorReader(bf)
    r.decode(4)
    with pytest.raises(hb.CorruptedData):
        r.decode(5)
