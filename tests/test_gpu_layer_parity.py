"""The benchmark's whole Llama-2-70B layer through the product decode against
the oracle, at the real shapes.

Every tensor of the layer (q/o 8192 x 8192, k/v 1024 x 8192, gate/up
28672 x 8192, down 8192 x 28672; N(0, 0.02), 1 % of columns x10, the bench's
seeds) is encoded by the oracle's writer (DCT-II, retention 0.30, INT4 with
FP16 block scales, 16 KiB LZ4 blocks) and decoded through ``HctReader``:
LZ4 -> rank directory -> spectral row pack -> tcgen05 DFT stages -> column
pack -> stages.  The f32 output must lie within max-abs 1e-3 and cosine
0.99999 of the oracle's CPU decode of the same file (LZ4 + dequantize_int4 +
bitmap scatter + f32 Makhoul IDCT, which restates dct.rs:311-337: columns,
then rows).  The bf16 output, which the bench times, must lie within the
same bound plus its own half-ulp (2^-8 |x|).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYER_70B = [  # (name, rows, cols), seed 2 * 100 + index as in bench.py
    ("q_proj", 8192, 8192), ("k_proj", 1024, 8192), ("v_proj", 1024, 8192),
    ("o_proj", 8192, 8192), ("gate_proj", 28672, 8192), ("up_proj", 28672, 8192),
    ("down_proj", 8192, 28672),
]
MAX_ABS = 1e-3
MIN_COS = 0.99999


def _cos(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


@pytest.mark.parametrize("idx", range(len(LAYER_70B)), ids=[t[0] for t in LAYER_70B])
def test_layer_tensor_matches_oracle(hb, dev, idx):
    import torch
    from oracle import hct as OH

    name, rows, cols = LAYER_70B[idx]
    w = OH.gen_weight((rows, cols), 2 * 100 + idx)
    f = OH.encode_spectral_q4(w, 0.30, version=1)
    del w
    ref = OH.decode_spectral_q4_cpu(f)
    ctx = hb.Context(0)
    r = hb.HctReader(f, ctx)
    got = r.decode(hb.F32)
    torch.cuda.synchronize(dev)
    g = got.cpu().numpy()
    del got
    err = float(np.abs(g - ref).max())
    cos = _cos(g, ref)
    assert err <= MAX_ABS and cos >= MIN_COS, (name, err, cos)
    del g
    gb = r.decode(hb.BF16).float().cpu().numpy()
    over = np.abs(gb - ref) - (MAX_ABS + np.abs(ref) * 2.0 ** -8)
    assert float(over.max()) <= 0.0, (name, float(np.abs(gb - ref).max()))
    assert _cos(gb, ref) >= MIN_COS, name
    r.close()
    ctx.close()
