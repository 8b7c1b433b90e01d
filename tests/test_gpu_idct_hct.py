"""IDCT contractions and the full HCT decode on the GPU.

Tolerance: max-abs error <= 1e-3 and cosine >= 0.99999
against the reference f32 result (our oracle's Makhoul IDCT) and the f64
truth.  bf16 output adds its own rounding: |err| <= 1e-3 + 2^-8 |x|."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-3
MIN_COS = 0.99999


def _cos(a, b):
    a = a.astype(np.float64).reshape(-1)
    b = b.astype(np.float64).reshape(-1)
    na, nb = np.sqrt((a * a).sum()), np.sqrt((b * b).sum())
    if na == 0 or nb == 0:
        return 1.0 if na == nb else 0.0
    return float((a * b).sum() / (na * nb))


def _check(got, ref, tag=""):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64)).max()
    cos = _cos(got, ref)
    assert err <= MAX_ABS and cos >= MIN_COS, f"{tag}: max-abs {err:.3e} cos {cos:.8f}"


def _weights_coeffs(orc, shape, seed):
    from oracle import hct as OH

    w = OH.gen_weight(shape, seed)
    return orc.dct_2d(w.reshape(shape))


@pytest.mark.parametrize("shape", [(4, 4), (8, 8), (1, 64), (64, 1), (1, 1), (33, 47), (5, 130),
                                   (128, 256), (129, 257), (300, 1000), (1024, 1024)])
def test_idct_2d_vs_oracle_and_truth(hb, orc, dev, shape):
    import torch

    c = _weights_coeffs(orc, shape, sum(shape))
    ref32 = orc.idct_2d(c)
    truth = orc.idct_2d_f64_truth(c)
    got = hb.idct_2d(torch.from_numpy(c).to(dev)).cpu().numpy()
    assert got.shape == shape
    _check(got, ref32, f"{shape} vs f32 oracle")
    _check(got, truth, f"{shape} vs f64 truth")


def test_idct_reference_c_decoder_vectors(hb, golden, dev):
    import torch

    for case in golden["ref_c_idct"]:
        x = np.array(case["input"], np.float32).reshape(case["rows"], case["cols"])
        ref = np.array(case["idct"], np.float32).reshape(x.shape)
        got = hb.idct_2d(torch.from_numpy(x).to(dev)).cpu().numpy()
        _check(got, ref, f"ref/c {x.shape}")


def test_idct_spec_vector(hb, golden, dev):
    import torch

    v = golden["spec_dct"]
    c = np.array(v["dct_coefficients"], np.float32).reshape(v["shape"])
    got = hb.idct_2d(torch.from_numpy(c).to(dev)).cpu().numpy()
    # reconstruction of 1..16 (spec 7.1) within fp16-operand accuracy of values up to 16
    assert np.abs(got - np.arange(1, 17, dtype=np.float32).reshape(4, 4)).max() < 16 * 2e-3


@pytest.mark.parametrize("dt", ["F16", "BF16"])
def test_idct_half_outputs(hb, orc, dev, dt):
    import torch

    c = _weights_coeffs(orc, (256, 512), 5)
    ref = orc.idct_2d(c)
    got = hb.idct_2d(torch.from_numpy(c).to(dev), out_dtype=getattr(hb, dt)).float().cpu().numpy()
    ulp = 2.0 ** -8 if dt == "BF16" else 2.0 ** -11
    assert (np.abs(got - ref) <= MAX_ABS + ulp * np.abs(ref)).all()
    assert _cos(got, ref) >= MIN_COS


def test_idct_full_size_properties(hb, dev):
    """28672 x 8192 (gate/up shape): orthonormality (Parseval) and linearity on device."""
    import torch

    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(28672, 8192, device=dev, generator=g) * 0.02
    y = hb.idct_2d(x)
    nx, ny = x.double().norm().item(), y.double().norm().item()
    assert abs(ny / nx - 1) < 1e-4
    del y
    # linearity on a smaller full-width slab
    a = x[:1024].contiguous()
    b = torch.randn(1024, 8192, device=dev, generator=g) * 0.02
    lhs = hb.idct_2d(2 * a + b)
    rhs = 2 * hb.idct_2d(a) + hb.idct_2d(b)
    assert (lhs - rhs).abs().max().item() < 1e-3


# ------------------------------------------------------------- HCT files

@pytest.mark.parametrize("shape,version", [((64, 96), 1), ((33, 47), 2), ((1, 4096), 1),
                                           ((4096,), 2), ((100, 1), 1), ((512, 1024), 2)])
def test_spectral_hct_decode_vs_oracle(hb, orc, shape, version):
    from oracle import hct as OH

    w = OH.gen_weight(shape, 21)
    f = OH.encode_spectral_q4(w, version=version)
    ref = OH.decode_spectral_q4_cpu(f).reshape(shape)
    r = (hb.HctReaderV2 if version == 2 else hb.HctReader)(f)
    assert r.shape == list(shape)
    payload = r.decompress_all().cpu().numpy()
    assert np.array_equal(payload, OH.decompress_all_cpu(OH.parse_hct(f)))
    got = r.decode(hb.F32).cpu().numpy()
    _check(got, ref, f"hct {shape}")
    bf = r.decode(hb.BF16).float().cpu().numpy()
    assert (np.abs(bf - ref) <= MAX_ABS + 2.0 ** -8 * np.abs(ref)).all()


def test_spectral_hct_config3_k_proj(hb, orc):
    """One BASELINE config-3 tensor (k_proj 1024 x 8192, seed 2) end to end vs the oracle."""
    from oracle import hct as OH

    w = OH.gen_weight((1024, 8192), 2)
    f = OH.encode_spectral_q4(w)
    ref = OH.decode_spectral_q4_cpu(f)
    got = hb.HctReader(f).decode(hb.F32).cpu().numpy()
    _check(got, ref, "k_proj")


def test_int4_hct_decode_bit_exact(hb, orc):
    from oracle import hct as OH

    for shape in [(64, 96), (1000,), (4096, 33)]:
        w = OH.gen_weight(shape, 3)
        f = OH.encode_int4_hct(w, version=2)
        ref = OH.decode_int4_hct_cpu(f).reshape(shape)
        got = hb.HctReaderV2(f).decode(hb.F32).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_container_errors(hb, orc):
    from oracle import hct as OH

    w = OH.gen_weight((64, 256), 4)
    f = bytearray(OH.encode_spectral_q4(w, version=2))
    bad = bytearray(f)
    bad[0] = ord("X")
    with pytest.raises(hb.CorruptedData, match="magic"):
        hb.HctReader(bytes(bad))
    bad = bytearray(f)
    bad[40] ^= 1
    with pytest.raises(hb.ChecksumMismatch, match="header checksum"):
        hb.HctReaderV2(bytes(bad))
    bad = bytearray(f)
    bad[-3] ^= 0x10
    with pytest.raises(hb.ChecksumMismatch, match="block"):
        hb.HctReaderV2(bytes(bad))
    bad = bytearray(f)
    bad[4] = 7  # version
    with pytest.raises(hb.CorruptedData, match="version"):
        hb.HctReader(bytes(bad))
    # a corrupt LZ4 block without checksums: same error variant as the oracle
    g = bytearray(OH.encode_spectral_q4(w, version=1))
    p = OH.parse_hct(bytes(g))
    start = len(g) - len(p.data)
    g[start] = 0x1F  # first token: 1 literal + extended match
    g[start + 2] = 0
    g[start + 3] = 0  # zero offset
    with pytest.raises(hb.CorruptedData, match="zero offset") as ei:
        hb.HctReader(bytes(g)).decode(hb.F32)
    assert ei.value.block == 0
    # the asynchronous form reports the same error from wait()
    import torch

    r = hb.HctReader(bytes(g))
    out = torch.empty(r.shape, dtype=torch.float32, device="cuda")
    r.decode_async(out, hb.F32)
    with pytest.raises(hb.CorruptedData, match="zero offset"):
        r.wait()


def test_async_decode_matches_sync(hb, orc):
    import torch
    from oracle import hct as OH

    files = [OH.encode_spectral_q4(OH.gen_weight(s, 50 + i)) for i, s in
             enumerate([(256, 512), (64, 1024), (512, 256)])]
    readers = [hb.HctReader(f) for f in files]
    outs = [torch.empty(r.shape, dtype=torch.float32, device="cuda") for r in readers]
    for r, o in zip(readers, outs):
        r.decode_async(o, hb.F32)
    for r in readers:
        r.wait()
    for r, o in zip(readers, outs):
        assert torch.equal(o, r.decode(hb.F32))


def test_upload_on_copy_stream_is_ordered(hb, orc):
    """upload() on a second stream waits for the previous decode's read of the
    buffer, and the next decode waits for the upload (no host sync between)."""
    import torch
    from oracle import hct as OH

    f = OH.encode_spectral_q4(OH.gen_weight((256, 1024), 77))
    ref = hb.HctReader(f).decode(hb.F32)
    r = hb.HctReader(f)
    hdr_len = len(f) - len(OH.parse_hct(f).data)
    zeros = bytes(f[:hdr_len]) + bytes(len(f) - hdr_len)  # same layout, data all zero
    pinned_f = torch.empty(len(f), dtype=torch.uint8, pin_memory=True)
    pinned_f.numpy()[:] = np.frombuffer(f, np.uint8)
    pinned_z = torch.empty(len(f), dtype=torch.uint8, pin_memory=True)
    pinned_z.numpy()[:] = np.frombuffer(zeros, np.uint8)
    comp, copy = torch.cuda.current_stream(), torch.cuda.Stream()
    out1 = torch.empty_like(ref)
    out2 = torch.empty_like(ref)
    out3 = torch.empty_like(ref)
    for _ in range(3):
        r.decode_async(out1, hb.F32, stream=comp)
        r.upload(pinned_z.numpy(), stream=copy)  # must not overwrite the data under decode 1
        r.wait()
        assert torch.equal(out1, ref)
        r.decode_async(out2, hb.F32, stream=comp)  # must see the zeros: a zero LZ4 offset
        with pytest.raises(hb.CorruptedData, match="zero offset"):
            r.wait()
        r.upload(pinned_f.numpy(), stream=copy)
        r.decode_async(out3, hb.F32, stream=comp)
        r.wait()
        assert torch.equal(out3, ref)
