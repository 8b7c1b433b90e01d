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


def makhoul_fold_table(P, Q, kbc):
    """The per-pair matrices of stage mode 6 (fdct.cu makhoul_fold_kernel), f64:
    (Q/2 + 1, 256, 128 kbc), rows 128 h + 2 m1 + ri, columns 64 kbc blk + r."""
    H = P * Q
    L = 2 * H
    KC = 64 * kbc
    T = np.zeros((Q // 2 + 1, 256, 2 * KC))
    m1 = np.arange(P)
    for u in range(Q // 2 + 1):
        for h in (0, 1):
            if h == 1 and (u == 0 or 2 * u == Q):
                continue
            k2 = Q - u if h else u
            for blk in (0, 1):
                for r in range(2 * P):
                    if blk == h:
                        role, k1 = (0, r) if r < P else (2, r - P)
                    elif k2 != 0:
                        role, k1 = (3, P - 1 - r) if r < P else (1, 2 * P - 1 - r)
                    elif r != 0:
                        role, k1 = (3, P - r) if r <= P else (1, 2 * P - r)
                    else:
                        continue
                    k = Q * k1 + k2
                    if role <= 1:
                        w = 1 / np.sqrt(2.0) if k == 0 else 0.5
                        coef = w * np.exp(1j * np.pi * k / (2 * L)) * (1 + 1j * np.exp(2j * np.pi * k / L))
                    else:
                        coef = 0.5 * np.exp(1j * np.pi * (k + H) / (2 * L)) * (1 - 1j * np.exp(2j * np.pi * k / L))
                    if role in (1, 3):
                        coef = -1j * coef
                    C = np.exp(2j * np.pi * ((m1 * k) % H) / H) * coef
                    T[u, 128 * h + 2 * m1, KC * blk + r] = C.real
                    T[u, 128 * h + 2 * m1 + 1, KC * blk + r] = C.imag
    return T


def stage1_fold(c, P, Q):
    """Lines c (B, L) -> G[m1][b][k2] the way stage mode 6 computes it: the
    lines read as T'[b][k2][r] = c[b][Q r + k2], pair u's tile multiplies
    columns u and (Q - u) mod Q by the pair's matrix (no pack)."""
    B, L = c.shape
    kbc = (2 * P + 63) // 64
    KC = 64 * kbc
    tab = makhoul_fold_table(P, Q, kbc)
    Tp = np.zeros((B, Q, KC))
    Tp[:, :, : 2 * P] = c.reshape(B, 2 * P, Q).transpose(0, 2, 1)
    G = np.zeros((P, B, Q), dtype=complex)
    for u in range(Q // 2 + 1):
        X = np.concatenate([Tp[:, u, :], Tp[:, (Q - u) % Q, :]], axis=1)  # (B, K)
        D = tab[u] @ X.T  # (256, B)
        G[:, :, u] = D[0 : 2 * P : 2] + 1j * D[1 : 2 * P : 2]
        if u != 0 and 2 * u != Q:
            G[:, :, Q - u] = D[128 : 128 + 2 * P : 2] + 1j * D[129 : 129 + 2 * P : 2]
    return G


@pytest.mark.parametrize("L,P,Q", [(8192, 64, 64), (4096, 32, 64), (14336, 56, 128),
                                   (256, 32, 4), (512, 32, 8)])
def test_makhoul_fold_matches_dct_iii(L, P, Q):
    """Stage mode 6 (Makhoul pack and twiddle folded into per-pair matrices)
    followed by stage 2 is the orthonormal DCT-III of the lines."""
    c = np.random.default_rng(L + 7).standard_normal((3, L))
    y = stage2(stage1_fold(c, P, Q), P, Q, L)
    ref = scipy.fft.idct(c, type=2, norm="ortho", axis=1)
    assert np.abs(y.T - ref).max() < 1e-9 * np.sqrt(L)


def test_line_slot_permutation_feeds_the_fold():
    """The row pass writes line b at slot (b % Q) 2P + b // Q (fdct.cu line_slot);
    its transposed output row n is then T'[n][k2][r] = x_n[Q r + k2]."""
    P, Q = 4, 8
    M = 2 * P * Q
    x = np.arange(M * 3).reshape(M, 3)  # x[b][n]: column n is the line of the next pass
    slot = (np.arange(M) % Q) * 2 * P + np.arange(M) // Q
    Tt = np.empty((3, M), dtype=x.dtype)
    Tt[:, slot] = x.T
    Tp = Tt.reshape(3, Q, 2 * P)
    for n in range(3):
        for k2 in range(Q):
            for r in range(2 * P):
                assert Tp[n, k2, r] == x[Q * r + k2, n]
