"""The torch writer (haagenti_b200/encode_gpu.py: float64 DCT-II, exact radix
select, quantize_int4, LZ4 HCT) against the oracle writer with its float64
DCT: byte-identical files.  Runs on the CPU here (the writer's torch code is
device-agnostic) and on the GPU in the gpu-marked case."""
import numpy as np
import pytest

from oracle import hct as OH

SHAPES = [((256, 512), 1), ((64, 1000), 2), ((1, 4096), 3), ((333, 96), 4), ((7, 9), 5),
          ((1, 33), 6)]


def _both(shape, seed, device, ratio=0.3):
    import torch

    from haagenti_b200 import encode_gpu as G

    w = OH.gen_weight(shape, seed)
    ref = OH.encode_spectral_q4(w, ratio, version=1, dct="f64")
    got = G.encode_spectral_q4_gpu(torch.from_numpy(w).to(device), ratio, version=1)
    return got, ref


@pytest.mark.parametrize("shape,seed", SHAPES)
def test_torch_writer_matches_oracle_writer_cpu(shape, seed):
    got, ref = _both(shape, seed, "cpu")
    assert got == ref


@pytest.mark.parametrize("ratio", [0.02, 0.5, 1.0])
def test_torch_writer_retention_cpu(ratio):
    got, ref = _both((96, 128), 9, "cpu", ratio)
    assert got == ref


def test_quantize_matches_oracle_on_edge_values():
    """Half-way quotients, zero blocks, a partial last block and an odd count."""
    import torch

    import oracle
    from haagenti_b200 import encode_gpu as G

    rng = np.random.default_rng(3)
    v = rng.standard_normal(32 * 9 + 5).astype(np.float32)
    v[32:64] = 0.0                                   # max|x| = 0 -> scale 1.0
    v[64:96] = np.float32(7.0) * np.arange(-16, 16) / np.float32(2.0)  # x / scale = k + 0.5
    v[96:128] = 1e-12                                # below the 1e-10 floor
    got = G.quantize_int4_gpu(torch.from_numpy(v)).numpy()
    assert np.array_equal(got, oracle.quantize_int4_np(v))


@pytest.mark.gpu
@pytest.mark.parametrize("shape,seed", SHAPES[:4])
def test_torch_writer_matches_oracle_writer_gpu(dev, shape, seed):
    got, ref = _both(shape, seed, dev)
    assert got == ref
