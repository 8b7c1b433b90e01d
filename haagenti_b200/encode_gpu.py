"""Writer side on the GPU: HCT-Q4 files of whole models at device speed.

The same encoder as ``encode.encode_spectral_q4`` (the counterparts of the
reference's encoder-side functions), with the heavy steps on the GPU:

* the orthonormal 2-D DCT-II (haagenti_core::dct::dct_2d,
  crates/haagenti-core/src/dct.rs:282-308) computed in float64 with the
  Makhoul FFT reordering and rounded once to float32, i.e. the correctly
  rounded coefficients;
* the retention of CompressiveSpectralEncoder::encode_2d
  (crates/haagenti/src/compressive.rs:140-172): the
  ``((n as f32 * ratio) as usize).max(1)`` largest |c|, ties to the lower
  index, as an LSB-first bitmap with the values in index order (an exact
  radix select on the float bit patterns);
* quantize_int4 (crates/haagenti/src/testing/quantization.rs:30-70): per 32
  values scale = max|x| / 7 (1.0 if <= 1e-10) stored as the truncating,
  flush-to-zero f16, q = x / scale rounded half away from zero and clamped
  to [-8, 7], nibble q + 8, low nibble first.

Only the LZ4 blocks and the container are made on the host (the library's
compress_block port, ``encode.write_hct``).  Given the same float32 weights,
the file is byte-identical to the oracle writer's with its float64 DCT
(``oracle.hct.encode_spectral_q4(..., dct="f64")``).

Not timed by the benchmark: it makes the decoder's inputs.
"""
from __future__ import annotations

import math

import numpy as np

from . import encode as E


def _torch():
    import torch

    return torch


def _dct_last_f64(x):
    """Orthonormal DCT-II along the last axis of a float64 CUDA tensor (Makhoul:
    v = even samples ascending ++ odd samples descending, X_k = Re(e^{-i pi k/2N} V_k))."""
    torch = _torch()
    n = x.shape[-1]
    v = torch.cat([x[..., 0::2], x[..., 1::2].flip(-1)], dim=-1)
    V = torch.fft.fft(v, dim=-1)
    del v
    k = torch.arange(n, device=x.device, dtype=torch.float64)
    ang = -math.pi * k / (2.0 * n)
    X = V.real * torch.cos(ang) - V.imag * torch.sin(ang)
    del V
    X *= math.sqrt(2.0 / n)
    X[..., 0] *= math.sqrt(0.5)
    return X


def dct_2d_gpu(w):
    """float32 (rows, cols) CUDA tensor -> its orthonormal 2-D DCT-II, float32
    (computed in float64, rounded once)."""
    x = w.double()
    x = _dct_last_f64(x)                      # along rows (length cols)
    x = _dct_last_f64(x.t().contiguous()).t()  # along columns (length rows)
    return x.float().contiguous()


def _f32_to_f16_trunc(v):
    """quantization.rs:136-163 on a float32 CUDA tensor -> int32 holding the f16 bits."""
    torch = _torch()
    b = v.contiguous().view(torch.int32)
    sign = (b >> 31) & 1
    exp = (b >> 23) & 0xFF
    frac = b & 0x7FFFFF
    ne = exp - 127 + 15
    out = sign << 15
    inf_nan = exp == 0xFF
    out = torch.where(inf_nan, (sign << 15) | (0x1F << 10) | (frac >> 13), out)
    normal = (exp != 0) & ~inf_nan
    out = torch.where(normal & (ne >= 31), (sign << 15) | (0x1F << 10), out)
    ok = normal & (ne > 0) & (ne < 31)
    out = torch.where(ok, (sign << 15) | (ne.clamp(0, 31) << 10) | (frac >> 13), out)
    return out


def quantize_int4_gpu(vals):
    """quantize_int4 of a float32 CUDA vector -> uint8 CUDA tensor
    (ceil(n/32) f16 LE scales, then ceil(n/2) nibble bytes)."""
    torch = _torch()
    n = vals.numel()
    if n == 0:
        return torch.zeros(0, dtype=torch.uint8, device=vals.device)
    nb = (n + 31) // 32
    pad = torch.zeros(nb * 32, dtype=torch.float32, device=vals.device)
    pad[:n] = vals
    blocks = pad.view(nb, 32)
    max_abs = blocks.abs().amax(dim=1)
    scale = torch.where(max_abs > 1e-10, max_abs / 7.0, torch.ones_like(max_abs))
    h = _f32_to_f16_trunc(scale)
    scales = torch.stack([h & 0xFF, (h >> 8) & 0xFF], dim=1).to(torch.uint8).reshape(-1)
    v = blocks / scale[:, None]          # IEEE f32 division, as x / scale
    t = torch.trunc(v)
    r = t + torch.where((v - t).abs() >= 0.5, torch.sign(v), torch.zeros_like(v))
    q = r.clamp(-8, 7).to(torch.int32).reshape(-1)[:n] + 8
    if n & 1:
        q = torch.cat([q, torch.zeros(1, dtype=torch.int32, device=q.device)])
        q[-1] = 0  # the missing high nibble of the last byte is zero
    nib = (q[0::2] | (q[1::2] << 4)).to(torch.uint8)
    return torch.cat([scales, nib])


def retain_count(n: int, ratio: float) -> int:
    return E.retain_count(n, ratio)


def spectral_select_gpu(coeffs, ratio: float = 0.30):
    """(bitmap uint8 CUDA tensor, retained float32 values in index order)."""
    torch = _torch()
    c = coeffs.reshape(-1)
    n = c.numel()
    k = min(retain_count(n, ratio), n)
    bits = c.abs().view(torch.int32)
    # largest T with count(bits >= T) >= k (bit order = value order for |c|)
    lo, hi = 0, 0x7F800000
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if int(torch.count_nonzero(bits >= mid)) >= k:
            lo = mid
        else:
            hi = mid - 1
    T = lo
    mask = bits > T
    need = k - int(torch.count_nonzero(mask))
    if need > 0:
        eq = torch.nonzero(bits == T).reshape(-1)[:need]  # lowest indices first
        mask[eq] = True
    nbytes = (n + 7) // 8
    m8 = torch.zeros(nbytes * 8, dtype=torch.uint8, device=c.device)
    m8[:n] = mask.to(torch.uint8)
    weights = (1 << torch.arange(8, device=c.device, dtype=torch.int32))
    bitmap = (m8.view(nbytes, 8).to(torch.int32) * weights).sum(dim=1).to(torch.uint8)
    return bitmap, c[mask]


def spectral_payload_gpu(w, ratio: float = 0.30):
    """bitmap ++ quantize_int4(retained) of a (rows, cols) float32 CUDA tensor, on the
    device."""
    torch = _torch()
    c = dct_2d_gpu(w)
    bitmap, vals = spectral_select_gpu(c, ratio)
    del c
    return torch.cat([bitmap, quantize_int4_gpu(vals)])


def encode_spectral_q4_gpu(w, ratio: float = 0.30, version: int = 1, shape=None) -> bytes:
    """HCT-Q4 file of a float32 CUDA tensor (rows, cols); ``shape`` is the shape
    recorded in the header (default: w's)."""
    payload = spectral_payload_gpu(w, ratio).cpu().numpy()
    return E.write_hct(payload, list(shape if shape is not None else w.shape), E.DTYPE_I4,
                       E.FLAG_SPECTRAL_Q4, version)


def synthetic_weight_gpu(shape, seed: int, device, outlier_frac: float = 0.01,
                         std: float = 0.02):
    """Seeded N(0, std) float32 weights made on the GPU (torch's Philox generator
    seeded with ``seed``); for 2-D shapes the first 1% of a default_rng([seed, 1])
    column permutation is scaled x10."""
    torch = _torch()
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    w = torch.randn(tuple(int(s) for s in shape), generator=g, device=device,
                    dtype=torch.float32)
    w *= std
    if outlier_frac > 0 and w.dim() == 2:
        nout = max(1, int(w.shape[1] * outlier_frac))
        cols = np.random.default_rng([seed, 1]).permutation(w.shape[1])[:nout]
        w[:, torch.from_numpy(cols).to(device)] *= 10.0
    return w
