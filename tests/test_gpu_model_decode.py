"""A whole (small) model through the loader pattern the bench times: every
tensor encoded on the GPU by the torch writer, decoded by HctReader.decode_async
on two decode contexts with statuses read back a window behind, each output
checked against the oracle's CPU decode of the same file."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# a Llama-shaped model small enough for the oracle: the 1000-long vocabulary
# axis (H = 500 = 5 x 100) takes the padded pack
TINY = dict(layers=3, hidden=256, intermediate=512, heads=4, kv_heads=2, head_dim=64,
            vocab=1000)


def _cos(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


def test_tiny_model_windowed_decode_matches_oracle(hb, dev):
    import torch
    from collections import deque

    from haagenti_b200 import encode_gpu as G
    from haagenti_b200 import shard
    from oracle import hct as OH

    units = shard.model_units(TINY)
    assert sum(1 for _ in units) == 3 * 9 + 3
    files = {}
    for i, (name, shape, _) in enumerate(units):
        w = G.synthetic_weight_gpu(shape, 5 * 100000 + i, dev)
        rows, cols = (1, shape[0]) if len(shape) == 1 else shape
        files[name] = G.encode_spectral_q4_gpu(w.reshape(rows, cols), 0.30, shape=shape)
    ctxs = (hb.Context(0), hb.Context(0))
    streams = (torch.cuda.current_stream(dev), torch.cuda.Stream(dev))
    readers = {n: hb.HctReader(files[n], ctxs[i % 2]) for i, (n, _, _) in enumerate(units)}
    outs = {n: torch.empty(s, dtype=torch.bfloat16, device=dev) for n, s, _ in units}
    f32 = {n: torch.empty(s, dtype=torch.float32, device=dev) for n, s, _ in units}
    for out_dtype, bufs in ((hb.BF16, outs), (hb.F32, f32)):
        pend = deque()
        for i, (n, _, _) in enumerate(units):
            readers[n].decode_async(bufs[n], out_dtype, stream=streams[i % 2])
            pend.append(readers[n])
            if len(pend) > 4:
                pend.popleft().wait()
        while pend:
            pend.popleft().wait()
    torch.cuda.synchronize(dev)
    for n, s, _ in units:
        ref = OH.decode_spectral_q4_cpu(files[n]).reshape(s)
        g = f32[n].cpu().numpy()
        assert float(np.abs(g - ref).max()) <= 1e-3, n
        assert _cos(g, ref) >= 0.99999, n
        gb = outs[n].float().cpu().numpy()
        assert float((np.abs(gb - ref) - (1e-3 + np.abs(ref) * 2.0 ** -8)).max()) <= 0.0, n
    for r in readers.values():
        r.close()
    for c in ctxs:
        c.close()
