"""The factored IDCT (Makhoul pack + two tcgen05 DFT stages per axis) against
the oracle, the f64 truth and the dense-basis contraction.  Tolerance as in
test_gpu_idct_hct.py: max-abs <= 1e-3, cosine >= 0.99999."""
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


def _coeffs(orc, shape, seed):
    from oracle import hct as OH

    return orc.dct_2d(OH.gen_weight(shape, seed).reshape(shape))


@pytest.fixture(scope="module")
def ctxs(hb):
    auto = hb.Context(0)
    dense = hb.Context(0)
    dense.set_idct(hb.IDCT_DENSE)
    return auto, dense


@pytest.mark.parametrize("shape", [(32, 32), (64, 128), (128, 96), (512, 256), (768, 4608),
                                   (1024, 1024), (1, 8192), (8192, 1), (1024, 8192),
                                   (8192, 8192)])
def test_factored_vs_oracle_truth_and_dense(hb, orc, dev, ctxs, shape):
    import torch

    auto, dense = ctxs
    c = _coeffs(orc, shape, 7 + sum(shape))
    x = torch.from_numpy(c).to(dev)
    got = hb.idct_2d(x, ctx=auto).cpu().numpy()
    ref = orc.idct_2d(c)
    _check(got, ref, f"{shape} factored vs oracle f32")
    if c.size <= 1 << 22:
        _check(got, orc.idct_2d_f64_truth(c), f"{shape} factored vs f64")
    d = hb.idct_2d(x, ctx=dense).cpu().numpy()
    _check(got, d, f"{shape} factored vs dense")


def test_factored_full_gate_shape(hb, dev, ctxs):
    """28672 x 8192 (gate/up, P x Q = 112 x 128 along rows): dense vs factored, Parseval."""
    import torch

    auto, dense = ctxs
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(28672, 8192, device=dev, generator=g) * 0.02
    a = hb.idct_2d(x, ctx=auto)
    assert abs(a.double().norm().item() / x.double().norm().item() - 1) < 1e-4
    d = hb.idct_2d(x, ctx=dense)
    diff = (a - d).abs().max().item()
    assert diff < MAX_ABS, diff
    cos = torch.nn.functional.cosine_similarity(a.double().flatten(), d.double().flatten(), dim=0)
    assert cos.item() >= MIN_COS


@pytest.mark.parametrize("shape", [(1024, 8192), (8192, 1024), (4096, 14336), (256, 512),
                                   (320, 4608), (64, 28672),
                                   # column passes with the Makhoul pack folded into
                                   # stage 1 (2P = 128, 64 and 112 with Q = 128)
                                   (8192, 256), (4096, 384), (14336, 256)])
def test_factored_hct_decode(hb, orc, shape):
    from oracle import hct as OH

    w = OH.gen_weight(shape, 40)
    f = OH.encode_spectral_q4(w)
    ref = OH.decode_spectral_q4_cpu(f)
    got = hb.HctReader(f).decode(hb.F32).cpu().numpy()
    _check(got, ref, f"hct {shape}")


@pytest.mark.parametrize("retention", [0.02, 0.3, 0.6, 0.95, 1.0])
def test_factored_hct_decode_retention(hb, orc, retention):
    """Rows with few and with more than L/2 retained coefficients: the fused
    row pack stages fp16 values for sparse rows and raw nibbles for dense ones."""
    from oracle import hct as OH

    shape = (192, 2048)
    w = OH.gen_weight(shape, 41)
    f = OH.encode_spectral_q4(w, retention=retention)
    ref = OH.decode_spectral_q4_cpu(f)
    for dt, tol in ((hb.F32, 0.0), (hb.BF16, 2.0 ** -8)):
        got = hb.HctReader(f).decode(dt).float().cpu().numpy()
        err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        assert (err <= MAX_ABS + tol * np.abs(ref)).all(), f"retention {retention}: {err.max():.3e}"
        assert _cos(got, ref) >= MIN_COS


@pytest.mark.parametrize("shape", [(32000, 64), (64, 32000), (128256, 64), (42752, 16),
                                   (96, 80), (80, 96)])
def test_factored_vocabulary_lengths(hb, orc, dev, ctxs, shape):
    """Axis lengths whose half has no split into two multiples of 4 up to 128:
    32000 (H = 125 x 128, Llama-2's vocabulary), 128256 (H = 501 x 128,
    Llama-3's; stage 1 on the tiled contraction), 42752 (H = 167 x 128) and 80
    (H = 1 x 40).  Through the reader (spectral payload -> factored IDCT) against
    the oracle's decode of the same file, and the bare IDCT against the dense
    contraction where its basis is small."""
    import torch
    from oracle import hct as OH

    w = OH.gen_weight(shape, 43)
    f = OH.encode_spectral_q4(w)
    ref = OH.decode_spectral_q4_cpu(f)
    got = hb.HctReader(f).decode(hb.F32).cpu().numpy()
    _check(got, ref, f"hct {shape}")
    auto, dense = ctxs
    if max(shape) <= 42752:
        c = OH.decode_spectral_q4_cpu(f, stage="coeffs")
        x = torch.from_numpy(np.ascontiguousarray(c)).to(dev)
        a = hb.idct_2d(x, ctx=auto).cpu().numpy()
        _check(a, ref, f"idct {shape} factored vs oracle")
        if max(shape) <= 32000:
            _check(a, hb.idct_2d(x, ctx=dense).cpu().numpy(), f"idct {shape} factored vs dense")
