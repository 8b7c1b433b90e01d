"""The C-ABI library loads and exports exactly what include/hct_b200.h declares.
No compute calls: these run without a GPU."""
import ctypes as C
import os
import re

import pytest

from haagenti_b200 import _lib as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(REPO, "include", "hct_b200.h")).read()
    return sorted(set(re.findall(r"\b(hct_b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_symbols()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(L.SIGNATURES) == names


def test_struct_layouts_match_header(tmp_path):
    """ctypes mirrors == what a C compiler makes of include/hct_b200.h."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    src = tmp_path / "sz.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "hct_b200.h"\n'
        'int main(void){printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(hct_b200_lz4_block),'
        ' sizeof(hct_b200_status), sizeof(hct_b200_header), sizeof(hct_b200_error),'
        ' offsetof(hct_b200_header, shape), offsetof(hct_b200_error, message));return 0;}')
    exe = tmp_path / "sz"
    subprocess.run([cc, "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                           check=True).stdout.split()]
    assert got == [C.sizeof(L.Lz4Block), C.sizeof(L.BlockStatus), C.sizeof(L.Header),
                   C.sizeof(L.Error), L.Header.shape.offset, L.Error.message.offset]


def test_status_strings_and_abi():
    lib = L.load()
    assert lib.hct_b200_abi_version() == 2
    assert lib.hct_b200_status_string(L.BUFFER_TOO_SMALL) == b"buffer too small"
    assert lib.hct_b200_status_string(L.ZERO_OFFSET).endswith(b"invalid zero offset")


def test_no_device_is_an_error_not_a_fallback():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = L.load()
    h = C.c_void_p()
    assert lib.hct_b200_ctx_create(0, C.byref(h)) == L.NO_DEVICE
    assert not h.value


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "absent.so"))
    monkeypatch.setattr(L, "_lib", None)
    with pytest.raises(ImportError, match="no CPU fallback"):
        L.load()


def test_rust_sys_crate_declares_every_header_symbol():
    """The Rust binding (rust/haagenti-b200-sys, not compiled here: no Rust
    toolchain) declares exactly the functions the header declares."""
    import re

    hdr = open(os.path.join(REPO, "include", "hct_b200.h")).read()
    rs = open(os.path.join(REPO, "rust", "haagenti-b200-sys", "src", "lib.rs")).read()
    want = set(re.findall(r"\b(hct_b200_[a-z0-9_]+)\s*\(", hdr))
    got = set(re.findall(r"pub fn (hct_b200_[a-z0-9_]+)\(", rs))
    assert got == want
