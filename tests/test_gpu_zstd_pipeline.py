"""ZstdGpuPipeline, the reference's GPU zstd pipeline interface
(crates/haagenti-cuda/src/zstd_gpu.rs:348-402), on the GPU decoder; the
cases follow the reference's pipeline tests (zstd_gpu.rs:860-1026):
simple, large, batch, to-GPU, empty, highly compressible, random, invalid
input.  Frames are written by libzstd at level 3, as ``zstd::encode_all``."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _z(d, level=3):
    from oracle import zstd_ref as Z

    return Z.compress(d, level)


def test_pipeline_simple_and_large_frames(hb):
    p = hb.ZstdGpuPipeline()
    assert p.is_ready()
    small = b"tensor weights, compressed and decoded on the device " * 40
    assert p.decompress(_z(small)) == small
    rng = np.random.default_rng(11)
    large = (rng.standard_normal(3_000_000) * 0.02).astype(np.float16).tobytes()
    assert p.decompress(_z(large)) == large


def test_pipeline_batch(hb):
    p = hb.ZstdGpuPipeline()
    originals = [f"fragment {i}: ".encode() * (50 + 37 * i) for i in range(10)]
    frames = [_z(d) for d in originals]
    from oracle import zstd_ref as Z

    frames[3] = Z.compress(originals[3], 3, content_size=False)  # decoded on its own
    res = p.decompress_batch(frames)
    assert len(res) == 10
    for r, d in zip(res, originals):
        assert r == d


def test_pipeline_to_gpu(hb, dev):
    p = hb.ZstdGpuPipeline()
    rng = np.random.default_rng(12)
    d = rng.integers(0, 16, 200_000, dtype=np.uint8).tobytes()
    t = p.decompress_to_gpu(_z(d))
    assert t.device.type == "cuda" and t.numel() == len(d)
    assert t.cpu().numpy().tobytes() == d


def test_pipeline_empty_random_compressible(hb):
    p = hb.ZstdGpuPipeline()
    assert p.decompress(_z(b"")) == b""
    zeros = bytes(1 << 20)
    c = _z(zeros)
    assert len(c) < len(zeros) // 10
    assert p.decompress(c) == zeros
    rnd = np.random.default_rng(13).integers(0, 256, 300_000, dtype=np.uint8).tobytes()
    assert p.decompress(_z(rnd)) == rnd


def test_pipeline_invalid_and_dictionary(hb):
    p = hb.ZstdGpuPipeline()
    with pytest.raises(hb.HaagentiError):
        p.decompress(b"not a zstd frame at all")
    with pytest.raises(hb.Unsupported):
        p.decompress_with_dict(_z(b"abc"), b"dictionary")
