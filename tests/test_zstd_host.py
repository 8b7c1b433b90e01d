"""The GPU Zstandard decoder's logic on the CPU: haagenti_b200/csrc/zstd_core.cuh
built as plain C++ (one lane) by g++ and checked against libzstd, the library
the reference's `zstd` crate binds (tests/zstd_host_check.cpp): libzstd's
bytes on every valid frame; the block-parallel plan agreeing with the serial
decode; an error wherever libzstd reports one on corrupted frames."""
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _libzstd() -> str | None:
    for d in ("/usr/lib/x86_64-linux-gnu", "/usr/lib64", "/usr/lib", "/lib/x86_64-linux-gnu"):
        p = os.path.join(d, "libzstd.so.1")
        if os.path.exists(p):
            return p
    return None


@pytest.mark.skipif(shutil.which("g++") is None or _libzstd() is None,
                    reason="needs g++ and the system libzstd")
def test_host_decoder_against_libzstd():
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "zstd_host_check")
        subprocess.run(["g++", "-O2", "-std=c++17", "-Wall",
                        os.path.join(HERE, "zstd_host_check.cpp"), "-o", exe, _libzstd()],
                       check=True, timeout=300)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    last = r.stdout.strip().splitlines()[-1].split()
    stats = dict(zip(last[0::2], map(int, last[1::2])))
    assert stats["failures"] == 0
    assert stats["cases"] > 1500
    # the block-parallel path is exercised, with and without sequence blocks
    assert stats["planned_decoded"] > 500
    # strictness beyond libzstd stays rare (corrupted Huffman stream ends)
    assert stats["stricter"] < stats["cases"] // 20
