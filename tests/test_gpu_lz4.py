"""LZ4 on the GPU (warp-per-block kernel) against the CPU oracle: bit-exact
output and identical error variant / position for every block."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _blocks_for(payloads, comps, capacities=None, sizes=None):
    d = np.zeros(len(comps), dtype=[("src_off", "<u8"), ("dst_off", "<u8"), ("src_len", "<u4"),
                                    ("dst_cap", "<u4"), ("out_size", "<u4"), ("pad", "<u4")])
    so = do = 0
    for i, (p, c) in enumerate(zip(payloads, comps)):
        cap = len(p) if capacities is None else capacities[i]
        osz = len(p) if sizes is None else sizes[i]
        d[i] = (so, do, len(c), cap, osz, 0)
        so += len(c)
        do += cap
    return d, so, do


def test_reference_roundtrips_host_api(hb, orc, golden):
    dec = hb.Lz4Decompressor()
    assert dec.algorithm() == "lz4"
    for name, hexdata in golden["lz4_roundtrip"].items():
        data = bytes.fromhex(hexdata)
        comp = orc.lz4_compress_block(data)
        assert dec.decompress_with_size(comp, len(data)) == data, name
        buf = bytearray(len(data))
        assert dec.decompress_to(comp, buf) == len(data) and bytes(buf) == data
        # interop blocks from another LZ4 implementation
        assert dec.decompress_with_size(bytes.fromhex(golden["lz4_interop"][name]), len(data)) == data
        # unknown size: 4x guess, doubling only on BufferTooSmall (decompress.rs:33-57).
        # A complete block decoded with a larger guess ends in UnexpectedEof in the
        # reference; the GPU path must give the same outcome as the oracle.
        guess = 4 * len(comp)
        ref = orc.lz4_decompress_block(comp, guess)
        if ref.code == 0:
            assert dec.decompress(comp) == ref.data
        elif ref.code != 2:
            with pytest.raises(hb.HaagentiError) as ei:
                dec.decompress(comp)
            assert ei.value.code == ref.code and ei.value.position == ref.position


def test_error_semantics_match_oracle(hb, orc, golden):
    dec = hb.Lz4Decompressor()
    for case in golden["lz4_errors"]:
        blk = bytes.fromhex(case["block"])
        if case["capacity"] != case["output_size"]:
            continue
        if case["code"] == 0:
            got = dec.decompress_with_size(blk, case["output_size"])
            assert len(got) == case["written"], case["name"]
            continue
        with pytest.raises(hb.HaagentiError) as ei:
            dec.decompress_with_size(blk, case["output_size"])
        e = ei.value
        assert e.code == case["code"], case["name"]
        assert e.position == case["position"], case["name"]
        if case["code"] == 2:
            assert e.required == case["position"] and e.provided == case["provided"]


@pytest.mark.parametrize("staged", [True, False])
def test_batched_blocks_error_cases_device_api(hb, orc, golden, dev, staged):
    import torch

    cases = golden["lz4_errors"]
    comps = [bytes.fromhex(c["block"]) for c in cases]
    d, ssz, dsz = _blocks_for([b""] * len(cases), comps,
                              [c["capacity"] for c in cases], [c["output_size"] for c in cases])
    src = torch.from_numpy(np.frombuffer(b"".join(comps) + b"\0" * 16, np.uint8).copy()).to(dev)
    dst = torch.zeros(max(dsz, 1) + 16, dtype=torch.uint8, device=dev)
    st = hb.Lz4Decompressor().decompress_blocks(src, d, dst, staged=staged)
    for i, c in enumerate(cases):
        assert st["code"][i] == c["code"], c["name"]
        assert st["written"][i] == c["written"], c["name"]
        if c["code"]:
            assert st["position"][i] == c["position"], c["name"]
            assert st["provided"][i] == c["provided"], c["name"]


def _mixed_payloads(rng, count, max_len=70000):
    out = []
    for i in range(count):
        n = int(rng.integers(0, max_len))
        kind = i % 5
        if kind == 0:
            d = rng.integers(0, 256, n, dtype=np.uint8)
        elif kind == 1:
            d = rng.integers(0, 3, n, dtype=np.uint8)
        elif kind == 2:
            d = np.zeros(n, np.uint8)
        elif kind == 3:
            pat = rng.integers(0, 256, int(rng.integers(1, 40)), dtype=np.uint8)
            d = np.resize(pat, n)
        else:
            d = np.frombuffer((rng.standard_normal(n // 2 + 1) * 0.02).astype(np.float16).tobytes(),
                              np.uint8)[:n]
        out.append(d.tobytes())
    return out


@pytest.mark.parametrize("staged", [True, False])
def test_random_batches_bit_exact(hb, orc, dev, staged):
    import torch

    rng = np.random.default_rng(11)
    payloads = _mixed_payloads(rng, 300)
    comps = [orc.lz4_compress_block(p) for p in payloads]
    d, ssz, dsz = _blocks_for(payloads, comps)
    src = torch.from_numpy(np.frombuffer(b"".join(comps), np.uint8).copy()).to(dev)
    dst = torch.zeros(dsz + 16, dtype=torch.uint8, device=dev)
    st = hb.Lz4Decompressor().decompress_blocks(src, d, dst, staged=staged)
    assert (st["code"] == 0).all()
    assert (st["written"] == np.array([len(p) for p in payloads])).all()
    assert dst[:dsz].cpu().numpy().tobytes() == b"".join(payloads)


@pytest.mark.parametrize("staged", [True, False])
def test_corrupted_random_blocks_match_oracle(hb, orc, dev, staged):
    """Bit flips / truncations: same status as the oracle, same bytes when Ok."""
    import torch

    rng = np.random.default_rng(12)
    payloads = _mixed_payloads(rng, 200, 5000)
    comps = []
    for p in payloads:
        c = bytearray(orc.lz4_compress_block(p))
        if c:
            for _ in range(int(rng.integers(1, 4))):
                c[int(rng.integers(0, len(c)))] ^= 1 << int(rng.integers(0, 8))
            if rng.random() < 0.3:
                c = c[: int(rng.integers(0, len(c)))]
        comps.append(bytes(c))
    caps = [len(p) + int(rng.integers(0, 3)) for p in payloads]
    d, ssz, dsz = _blocks_for(payloads, comps, caps, caps)
    srcnp = np.frombuffer(b"".join(comps), np.uint8)
    ref_out, ref_st = orc.lz4_decompress_batch(srcnp, d.astype(orc.BLOCK_DESC), dsz)
    src = torch.from_numpy(srcnp.copy()).to(dev)
    dst = torch.zeros(dsz + 16, dtype=torch.uint8, device=dev)
    st = hb.Lz4Decompressor().decompress_blocks(src, d, dst, staged=staged)
    got = dst[:dsz].cpu().numpy()
    assert np.array_equal(st["code"], ref_st["code"])
    err = ref_st["code"] != 0
    assert np.array_equal(st["position"][err], ref_st["position"][err])
    assert np.array_equal(st["provided"][err], ref_st["aux"][err])
    for i in np.nonzero(~err)[0]:
        o = int(d["dst_off"][i])
        w = int(ref_st["written"][i])
        assert st["written"][i] == w
        assert np.array_equal(got[o:o + w], ref_out[o:o + w])


def test_config2_lz4_256mib_roundtrip(hb, orc, dev):
    """256 MiB of N(0,0.02) fp16 (seed 1) in 4096 x 64 KiB blocks."""
    import torch

    rng = np.random.default_rng(1)
    data = (rng.standard_normal(128 * 1024 * 1024, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    raw = data.view(np.uint8)
    packed, lens = orc.lz4_compress_chunks(raw, 65536)
    assert len(lens) == 4096
    d = np.zeros(4096, dtype=[("src_off", "<u8"), ("dst_off", "<u8"), ("src_len", "<u4"),
                              ("dst_cap", "<u4"), ("out_size", "<u4"), ("pad", "<u4")])
    d["src_off"][1:] = np.cumsum(lens[:-1], dtype=np.uint64)
    d["dst_off"] = np.arange(4096, dtype=np.uint64) * 65536
    d["src_len"] = lens
    d["dst_cap"] = 65536
    d["out_size"] = 65536
    src = torch.from_numpy(packed).to(dev)
    dst = torch.empty(raw.size, dtype=torch.uint8, device=dev)
    st = hb.Lz4Decompressor().decompress_blocks(src, d, dst)
    assert (st["code"] == 0).all() and (st["written"] == 65536).all()
    assert torch.equal(dst, torch.from_numpy(raw).to(dev))


def _lz4_len(n: int) -> bytes:
    out = bytearray()
    while n >= 255:
        out.append(255)
        n -= 255
    out.append(n)
    return bytes(out)


def _lz4_seq(lits: bytes, offset: int = 0, ml: int = 0) -> bytes:
    """One LZ4 sequence; offset == 0 makes it the literal-only last sequence."""
    ln = len(lits)
    mcode = ml - 4 if offset else 0
    tok = (min(ln, 15) << 4) | min(mcode, 15)
    out = bytearray([tok])
    if ln >= 15:
        out += _lz4_len(ln - 15)
    out += lits
    if offset:
        out += offset.to_bytes(2, "little")
        if mcode >= 15:
            out += _lz4_len(mcode - 15)
    return bytes(out)


@pytest.mark.parametrize("staged", [True, False])
def test_overlapping_matches_all_periods(hb, orc, dev, staged):
    """Crafted blocks whose matches overlap their source (offset < length) for
    periods 1..40 and large ones, at every output alignment: same bytes as the oracle."""
    import torch

    rng = np.random.default_rng(13)
    comps, sizes = [], []
    for period in list(range(1, 41)) + [63, 64, 65, 100, 255, 1000, 4097]:
        for lead in range(4):  # output alignment of the match
            lits = rng.integers(0, 256, lead + period, dtype=np.uint8).tobytes()
            # lead 3: outputs beyond 16 KiB from a small block (the staged
            # kernel decodes those straight in device memory)
            ml = int(rng.integers(period + 1, 9000 if lead < 3 else 60000))
            tail = rng.integers(0, 256, int(rng.integers(5, 40)), dtype=np.uint8).tobytes()
            blk = _lz4_seq(lits, period, ml) + _lz4_seq(tail)
            comps.append(blk)
            sizes.append(len(lits) + ml + len(tail))
    d, ssz, dsz = _blocks_for([b"\0" * n for n in sizes], comps)
    srcnp = np.frombuffer(b"".join(comps), np.uint8)
    ref_out, ref_st = orc.lz4_decompress_batch(srcnp, d.astype(orc.BLOCK_DESC), dsz)
    assert (ref_st["code"] == 0).all()
    src = torch.from_numpy(srcnp.copy()).to(dev)
    dst = torch.zeros(dsz + 16, dtype=torch.uint8, device=dev)
    st = hb.Lz4Decompressor().decompress_blocks(src, d, dst, staged=staged)
    assert (st["code"] == 0).all()
    assert np.array_equal(st["written"], ref_st["written"])
    assert np.array_equal(dst[:dsz].cpu().numpy(), ref_out[:dsz])


@pytest.mark.parametrize("staged", [False, True])
def test_long_literal_runs_every_alignment_phase(hb, orc, dev, staged):
    """Literal runs of 1 KiB and more (copied 16 bytes at a time from two
    aligned loads in the device-memory variant; from 2 KiB on through the
    bulk-copied shared-memory chunks of 4080 new bytes each, so lengths
    around one, two and three chunks are included) at every source-minus-
    destination offset mod 16 and several block starts: same bytes as the oracle."""
    import torch

    rng = np.random.default_rng(14)
    comps, sizes = [], []
    for run in (1024, 1031, 2063, 4079, 4097, 8161, 8200, 9001, 12241):
        for shift in range(16):
            for lead in (5, 6, 7, 8):
                head = rng.integers(0, 256, lead, dtype=np.uint8).tobytes()
                body = rng.integers(0, 256, run, dtype=np.uint8).tobytes()
                tail = rng.integers(0, 256, 9, dtype=np.uint8).tobytes()
                # the first match moves the output position by 4 + shift bytes
                # against the input position; the long run follows it
                blk = (_lz4_seq(head, 1, 4 + shift) + _lz4_seq(body, 3, 11)
                       + _lz4_seq(tail))
                comps.append(blk)
                sizes.append(lead + 4 + shift + run + 11 + len(tail))
    d, ssz, dsz = _blocks_for([b"\0" * n for n in sizes], comps)
    srcnp = np.frombuffer(b"".join(comps), np.uint8)
    ref_out, ref_st = orc.lz4_decompress_batch(srcnp, d.astype(orc.BLOCK_DESC), dsz)
    assert (ref_st["code"] == 0).all()
    src = torch.from_numpy(srcnp.copy()).to(dev)
    dst = torch.zeros(dsz + 16, dtype=torch.uint8, device=dev)
    st = hb.Lz4Decompressor().decompress_blocks(src, d, dst, staged=staged)
    assert (st["code"] == 0).all()
    assert np.array_equal(st["written"], ref_st["written"])
    assert np.array_equal(dst[:dsz].cpu().numpy(), ref_out[:dsz])
