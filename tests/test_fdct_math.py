"""The factored DCT-III that fdct.cu and the DFT-stage epilogues implement,
written out in numpy with the same index maps, pinned to scipy's
orthonormal DCT-III.  CPU only; documents the algorithm the kernels use."""
import numpy as np
import pytest
import scipy.fft


def pack(c, P, Q):
    """rows c (B, L) -> Z[b][k2][k1] (k = Q k1 + k2), as makhoul_pack_kernel."""
    B, L = c.shape
    H = L // 2
    c = c.astype(np.float64).copy()
    c[:, 0] /= np.sqrt(2.0)
    cm = np.zeros_like(c)
    cm[:, 1:] = c[:, :0:-1]  # c'[L-k], c'[L] = 0
    k = np.arange(L)
    V = np.where(k == 0, 1.0, 0.5) * (c - 1j * cm) * np.exp(1j * np.pi * k / (2 * L))
    kk = np.arange(H)
    Z = (V[:, :H] + V[:, H:]) + 1j * (V[:, :H] - V[:, H:]) * np.exp(2j * np.pi * kk / L)
    return Z.reshape(B, P, Q).transpose(0, 2, 1)


def stage1(Z, P, Q, H):
    """Z[b][k2][k1] -> G[m1][b][k2] (mode 2: DFT over k1, twiddle e^{2 pi i k2 m1 / H})."""
    W = np.exp(2j * np.pi * np.outer(np.arange(P), np.arange(P)) / P)
    G = np.einsum("ab,xqb->axq", W, Z)
    return G * np.exp(2j * np.pi * np.outer(np.arange(P), np.arange(Q)) / H)[:, None, :]


def stage2(G, P, Q, L):
    """G[m1][b][k2] -> Y[n][b] (mode 3: DFT over k2, j = m1 + P m2, quartet scatter)."""
    H = L // 2
    W = np.exp(2j * np.pi * np.outer(np.arange(Q), np.arange(Q)) / Q)
    z = np.einsum("ab,mxb->max", W, G)  # [m1][m2][b]
    zz = z.transpose(1, 0, 2).reshape(P * Q, -1) * np.sqrt(2.0 / L)  # [j][b]
    Y = np.empty((L, zz.shape[1]))
    j = np.arange(H)
    lo = j < H // 2
    Y[4 * j[lo]] = zz[lo].real
    Y[4 * j[lo] + 2] = zz[lo].imag
    Y[4 * (H - 1 - j[~lo]) + 3] = zz[~lo].real
    Y[4 * (H - 1 - j[~lo]) + 1] = zz[~lo].imag
    return Y


def axis(c, P, Q):
    L = c.shape[1]
    return stage2(stage1(pack(c, P, Q), P, Q, L // 2), P, Q, L)


@pytest.mark.parametrize("L,P,Q", [(32, 4, 4), (96, 12, 4), (128, 8, 8), (1024, 16, 32),
                                   (8192, 64, 64), (28672, 112, 128),
                                   # vocabulary lengths: P not a multiple of 4
                                   (32000, 125, 128), (128256, 501, 128), (80, 1, 40)])
def test_one_axis_matches_dct_iii(L, P, Q):
    c = np.random.default_rng(L).standard_normal((3, L))
    y = axis(c, P, Q)  # transposed: y[n][b]
    ref = scipy.fft.idct(c, type=2, norm="ortho", axis=1)
    assert np.abs(y.T - ref).max() < 1e-9 * np.sqrt(L)


def test_combined_pack_coefficients():
    """Z[k] = alpha_k (c[k] - i c[L-k]) + beta_k (c[H+k] - i c[H-k]), as pack_tables_kernel."""
    L, P, Q = 128, 8, 8
    H = L // 2
    c = np.random.default_rng(1).standard_normal((2, L))
    k = np.arange(H)
    a = np.exp(1j * np.pi * k / (2 * L))
    b = np.exp(1j * np.pi * (k + H) / (2 * L))
    t = np.exp(2j * np.pi * k / L)
    w = np.where(k == 0, 1 / np.sqrt(2.0), 0.5)
    alpha = w * a * (1 + 1j * t)
    beta = 0.5 * b * (1 - 1j * t)
    cL = np.where(k == 0, 0.0, c[:, (L - k) % L])
    Z = alpha * (c[:, k] - 1j * cL) + beta * (c[:, H + k] - 1j * c[:, H - k])
    ref = pack(c, P, Q).transpose(0, 2, 1).reshape(2, H)  # back to natural k order
    np.testing.assert_allclose(Z, ref, atol=1e-12)


def test_two_axes_give_idct_2d():
    # rows first (output T^T), then the rows of T^T (output X row-major)
    rng = np.random.default_rng(0)
    F = rng.standard_normal((64, 128))
    tt = axis(F, 8, 8)          # (128, 64) = T^T
    X = axis(tt, 4, 8)          # (64, 128)
    np.testing.assert_allclose(X, scipy.fft.idctn(F, type=2, norm="ortho"), atol=1e-10)
