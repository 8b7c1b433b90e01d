"""INT4 dequantisation on the GPU against the oracle: bit-exact f32, and
f16/bf16 equal to round-to-nearest-even of the exact f32 value."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


def test_config1_4096sq_bit_exact(hb, orc):
    """4096x4096 N(0,0.02), seed 0, 1% outlier columns x10."""
    from oracle import hct as OH

    w = OH.gen_weight((4096, 4096), 0)
    q = orc.quantize_int4_np(w.reshape(-1))
    assert q.size == 9_437_184
    ref = orc.dequantize_int4(q, w.size)
    got = hb.dequantize_int4(q, w.size).cpu().numpy()
    assert got.shape == ref.shape
    assert np.array_equal(_bits(got), _bits(ref))


@pytest.mark.parametrize("n", [1, 2, 7, 8, 9, 31, 32, 33, 63, 64, 65, 1000, 4097, 123457])
def test_ragged_sizes(hb, orc, n):
    rng = np.random.default_rng(n)
    w = (rng.standard_normal(n) * 0.05).astype(np.float32)
    q = orc.quantize_int4(w)
    ref = orc.dequantize_int4(q, n)
    got = hb.dequantize_int4(q, n).cpu().numpy()
    assert np.array_equal(_bits(got), _bits(ref))


def test_short_inputs_follow_reference_rules(hb, orc):
    n = 1000
    q = orc.quantize_int4((np.random.default_rng(1).standard_normal(n)).astype(np.float32))
    sb = 2 * ((n + 31) // 32)
    for cut in [0, 1, sb - 1, sb, sb + 1, sb + 7, len(q) - 1]:
        ref = orc.dequantize_int4(q[:cut], n)
        got = hb.dequantize_int4(q[:cut], n).cpu().numpy()
        assert got.size == ref.size, cut
        assert np.array_equal(_bits(got), _bits(ref)), cut
    assert hb.dequantize_int4(b"", 0).numel() == 0


def test_half_outputs(hb, orc):
    import torch

    n = 100_003
    w = (np.random.default_rng(2).standard_normal(n) * 3).astype(np.float32)
    q = orc.quantize_int4(w)
    ref = orc.dequantize_int4(q, n)
    f16 = hb.dequantize_int4(q, n, out_dtype=hb.F16).cpu()
    assert np.array_equal(f16.numpy().view(np.uint16), ref.astype(np.float16).view(np.uint16))
    bf = hb.dequantize_int4(q, n, out_dtype=hb.BF16).cpu()
    assert torch.equal(bf, torch.from_numpy(ref).to(torch.bfloat16))


def test_unaligned_device_buffers(hb, orc, dev):
    """Input at odd byte offsets, output at an odd element offset: same values."""
    import torch
    import ctypes as C
    from haagenti_b200 import _lib as L

    n = 4099
    w = (np.random.default_rng(3).standard_normal(n)).astype(np.float32)
    q = np.frombuffer(orc.quantize_int4(w), np.uint8)
    ref = orc.dequantize_int4(q, n)
    for off in range(4):
        buf = torch.zeros(q.size + 8, dtype=torch.uint8, device=dev)
        buf[off:off + q.size] = torch.from_numpy(q.copy()).to(dev)
        out = torch.zeros(n + 1, dtype=torch.float32, device=dev)
        written = C.c_size_t(0)
        rc = L.load().hct_b200_dequantize_int4(buf.data_ptr() + off, q.size, n,
                                               out.data_ptr() + 4, L.F32, C.byref(written),
                                               torch.cuda.current_stream().cuda_stream)
        assert rc == 0 and written.value == n
        got = out[1:].cpu().numpy()
        assert np.array_equal(_bits(got), _bits(ref)), off


def test_dequantize_int4_mp_vs_oracle(hb, orc):
    """mixed_precision.rs:489-539: bit-exact values, zero fill for short data."""
    import torch

    rng = np.random.default_rng(10)
    w = (rng.standard_normal(4099) * 0.02).astype(np.float32)
    q = orc.quantize_int4_mp(w)
    for cut in (len(q), len(q) - 1, 2 * 129 + 7, 2 * 129, 100, 1):
        ref = orc.dequantize_int4_mp(q[:cut], w.size)
        got = hb.dequantize_int4_mp(q[:cut], w.size).cpu().numpy()
        assert got.shape == ref.shape and np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        bf = hb.dequantize_int4_mp(q[:cut], w.size, hb.BF16).cpu()
        assert torch.equal(bf, torch.from_numpy(ref).to(torch.bfloat16))
    assert hb.dequantize_int4_mp(q, 0).numel() == 0
    assert hb.dequantize_int4_mp(b"", 10).numel() == 0


@pytest.mark.parametrize("n", [16384, 16385, 3 * 16384 + 5, 5 * 16384 - 8, 262144 + 31,
                               1_000_003])
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_staged_tiles_and_tails(hb, orc, dev, n, dt):
    """Sizes around the 16384-element tile of the bulk-staged path (whole tiles
    copied by cp.async.bulk, the partial last tile read directly), every output
    type: f32 bit-exact, f16/bf16 the RNE of that f32."""
    import torch

    rng = np.random.default_rng(n)
    w = (rng.standard_normal(n) * 0.05).astype(np.float32)
    q = orc.quantize_int4(w)
    ref = orc.dequantize_int4(q, n)
    code = {"f32": hb.F32, "f16": hb.F16, "bf16": hb.BF16}[dt]
    got = hb.dequantize_int4(torch.from_numpy(np.frombuffer(q, np.uint8).copy()).to(dev), n,
                             code).float().cpu().numpy()
    if dt == "f32":
        assert np.array_equal(_bits(got), _bits(ref))
    else:
        want = torch.from_numpy(ref).to(torch.float16 if dt == "f16" else torch.bfloat16)
        assert np.array_equal(got, want.float().numpy())


def test_batch_mixed_jobs_and_alignments(hb, orc, dev):
    """One batched call: jobs of many sizes, data at odd offsets (the direct-load
    path), outputs at offsets that rule out vector stores, short inputs and an
    empty job; every job bit-exact with its own dequantize_int4."""
    import torch

    rng = np.random.default_rng(5)
    sizes = [1, 33, 16384, 16384 * 2 + 7, 40000, 65536 * 3, 100001, 0, 70000]
    items, refs, outs = [], [], []
    for i, n in enumerate(sizes):
        w = (rng.standard_normal(n) * 0.03).astype(np.float32)
        q = np.frombuffer(orc.quantize_int4(w), np.uint8)
        if i == 8:
            q = q[: len(q) - 999]  # nibbles run out: fewer elements written
        off = [0, 2, 0, 6, 16, 0, 4, 0, 0][i]  # byte offset of the data in its buffer
        buf = torch.zeros(len(q) + off + 16, dtype=torch.uint8, device=dev)
        buf[off: off + len(q)] = torch.from_numpy(q.copy()).to(dev)
        items.append((buf[off: off + len(q)], n))
        refs.append(orc.dequantize_int4(q.tobytes(), n))
        o_off = [0, 1, 0, 3, 0, 0, 5, 0, 0][i]  # element offset of the output
        ob = torch.full((max(n, 1) + o_off,), float("nan"), dtype=torch.float32, device=dev)
        outs.append(ob[o_off:])
    got = hb.dequantize_int4_batch(items, hb.F32, outs=outs)
    for g, r, n in zip(got, refs, sizes):
        g = g.cpu().numpy()
        assert g.size == r.size, n
        assert np.array_equal(_bits(g), _bits(r)), n
