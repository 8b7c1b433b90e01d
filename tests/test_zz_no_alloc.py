"""The allocation-free spectral decode entry point.

Callers that cannot allocate device memory mid-decode (for example a serving
runtime whose allocator owns all of HBM) use
hct_b200_spectral_q4_decode_noalloc, whose scratch is a fixed array inside
the library.  This file checks, through the C ABI, that two calls in a row
give the same tensor as the context-based hct_b200_spectral_q4_decode, and
that requests beyond the array's limit are refused.  It is named so that
pytest collects it last."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-3
MIN_COS = 0.99999


def _payload(shape, seed):
    from oracle import hct as OH

    f = OH.encode_spectral_q4(OH.gen_weight(shape, seed))
    return OH.decompress_all_cpu(OH.parse_hct(f))


def _cos(a, b):
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return float((a * b).sum() / np.sqrt((a * a).sum() * (b * b).sum()))


def _decode_with_ctx(lib, ctx, d_payload, rows, cols, out, stream):
    return lib.hct_b200_spectral_q4_decode(ctx, d_payload.data_ptr(), d_payload.numel(), rows,
                                           cols, out.data_ptr(), 0, stream)


def _decode_noalloc(lib, d_payload, rows, cols, out, stream):
    return lib.hct_b200_spectral_q4_decode_noalloc(d_payload.data_ptr(), d_payload.numel(), rows,
                                                   cols, out.data_ptr(), 0, stream)


def test_noalloc_matches_context_decode_on_two_calls():
    import torch
    from haagenti_b200 import _lib as L

    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = L.load()
    ctx = C.c_void_p()
    assert lib.hct_b200_ctx_create(0, C.byref(ctx)) == 0
    stream = torch.cuda.current_stream(dev).cuda_stream
    try:
        cases = [((512, 1024), 31), ((300, 2048), 32)]
        refs, payloads = [], []
        for (rows, cols), seed in cases:
            p = torch.from_numpy(_payload((rows, cols), seed)).to(dev)
            ref = torch.empty((rows, cols), dtype=torch.float32, device=dev)
            assert _decode_with_ctx(lib, ctx, p, rows, cols, ref, stream) == 0
            refs.append(ref.cpu().numpy())
            payloads.append(p)
        # output buffers first, then one call to set up the scratch address on
        # this device, so that the free-memory reading below brackets only
        # the decodes themselves
        bufs = [torch.full((rows, cols), float("nan"), dtype=torch.float32, device=dev)
                for (rows, cols), _ in cases]
        warm = torch.empty(cases[0][0], dtype=torch.float32, device=dev)
        assert _decode_noalloc(lib, payloads[0], *cases[0][0], warm, stream) == 0
        torch.cuda.synchronize(dev)
        free_before = torch.cuda.mem_get_info(dev)[0]
        # two calls in a row through the shared scratch array, different shapes
        for ((rows, cols), _), p, out in zip(cases, payloads, bufs):
            assert _decode_noalloc(lib, p, rows, cols, out, stream) == 0
        torch.cuda.synchronize(dev)
        # the decodes took no device memory (cudaMemGetInfo unchanged)
        assert torch.cuda.mem_get_info(dev)[0] == free_before
        outs = [b.cpu().numpy() for b in bufs]
        for got, ref in zip(outs, refs):
            assert np.isfinite(got).all()
            assert np.abs(got - ref).max() <= MAX_ABS
            assert _cos(got, ref) >= MIN_COS
        # and the first shape again, after the second call left its data in the array
        (rows, cols), _ = cases[0]
        again = torch.empty((rows, cols), dtype=torch.float32, device=dev)
        assert _decode_noalloc(lib, payloads[0], rows, cols, again, stream) == 0
        assert np.abs(again.cpu().numpy() - refs[0]).max() <= MAX_ABS
    finally:
        lib.hct_b200_ctx_destroy(ctx)


def test_noalloc_rejects_tensors_beyond_its_scratch():
    import torch
    from haagenti_b200 import _lib as L

    dev = torch.device("cuda", 0)
    lib = L.load()
    p = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    out = torch.empty(16, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.hct_b200_spectral_q4_decode_noalloc(p.data_ptr(), p.numel(), 4096, 16,
                                                   out.data_ptr(), 0, stream) == L.INVALID_ARGUMENT
    assert lib.hct_b200_spectral_q4_decode_noalloc(p.data_ptr(), p.numel(), 16, 2049,
                                                   out.data_ptr(), 0, stream) == L.INVALID_ARGUMENT
