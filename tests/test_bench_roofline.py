"""The bench's roofline bookkeeping on CPU: every kernel record the 70B and
layer legs can name has exactly one traffic line in its committed profile
summary, and roofline_of turns per-launch event records into the line's
figures (achieved = algorithmic bytes / summed event time, frac against the
peak, step_hbm_frac over the uninstrumented step)."""
import os

import pytest

import bench

RECORDS = ["dft_stage1", "dft_stage2", "makhoul_pack", "spectral_pack"]


@pytest.mark.parametrize("path", [bench.MODEL_TRAFFIC_PROFILE, bench.TRAFFIC_PROFILE])
def test_profiles_carry_one_traffic_line_per_record(path):
    assert os.path.exists(path)
    lines = [l for l in open(path) if l.startswith("traffic_bytes_per_launch[")]
    keys = [l.split("]", 1)[0].split("[", 1)[1] for l in lines]
    assert len(keys) == len(set(keys)), f"duplicate traffic lines in {path}"
    for r in RECORDS:
        v = bench.read_traffic(r, path)
        assert v is not None and 1e7 < v < 1e10, (r, v)


def test_roofline_of_arithmetic():
    ks = {
        "dft_stage1": {"launches": 10, "ms": 2.0, "work": 4.0e9},
        "dft_stage2": {"launches": 10, "ms": 1.0, "work": 4.0e9},
        "spectral_pack": {"launches": 5, "ms": 1.5, "work": 1.0e9},
    }
    roof, kern = bench.roofline_of(ks, ms_prof=5.0, ms_per_step=4.0, steps=1,
                                   traffic_file=bench.MODEL_TRAFFIC_PROFILE)
    peak = bench.peaks()["hbm"]
    assert roof["bound"] == "hbm" and roof["kernel"] == bench.KERNEL_NAMES["dft_stage1"]
    assert roof["achieved"] == pytest.approx(4.0e9 / 2.0e-3 / 1e9)  # 2000 GB/s
    assert roof["frac"] == pytest.approx(2000.0 / peak, rel=1e-3)
    assert roof["algorithmic_per_launch"] == 4.0e8
    assert roof["share_of_step"] == pytest.approx(0.4)
    assert roof["traffic"] == bench.read_traffic("dft_stage1", bench.MODEL_TRAFFIC_PROFILE)
    assert roof["step_hbm_frac"] == pytest.approx(9.0e9 / 4.0e-3 / 1e9 / peak, rel=1e-3)
    assert kern["spectral_pack"]["rate"] == pytest.approx(1.0e9 / 1.5e-3 / 1e9, rel=1e-4)
