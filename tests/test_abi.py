"""The native library loads and exports every entry point its public headers declare
(CPU only: no compute call is made).

include/da3b.h and include/da3cpp/da3_c.h are C: every `DA3B_API` / `DA_CAPI`
function must be a dynamic symbol of libda3b.so with a ctypes signature in
da3cpplib_b200/_lib.py. include/da3cpp/da3.h is the C++ surface (namespace da3);
its `DA3_API` functions must be exported under their C++ names.
"""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")


def _declared(path, macro):
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"^\s*#[^\n]*", "", text, flags=re.M)
    return re.findall(macro + r"\s+[^;(]*?\**\s*\b([A-Za-z_]\w*)\s*\(", text)


def c_symbols():
    names = []
    for h, macro in (("da3b.h", "DA3B_API"), (os.path.join("da3cpp", "da3_c.h"), "DA_CAPI")):
        names += _declared(os.path.join(INC, h), macro)
    return names


@pytest.fixture(scope="module")
def so_path():
    from da3cpplib_b200 import _lib

    if not os.path.exists(_lib.LIB_PATH):
        pytest.fail("libda3b.so is not built (run __graft_entry__.build())")
    return _lib.LIB_PATH


def test_headers_declare_entry_points():
    names = c_symbols()
    assert len(names) >= 30
    assert "da3b_linear_f16" in names and "da_capi_load" in names and "da3b_attention" in names


def test_library_exports_every_c_symbol(so_path):
    lib = ctypes.CDLL(so_path)
    missing = [n for n in c_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_signatures_cover_headers():
    from da3cpplib_b200 import _lib

    missing = [n for n in c_symbols() if n not in _lib.SIGNATURES]
    assert not missing, f"no ctypes signature for: {missing}"


def test_library_exports_cpp_api(so_path):
    if shutil.which("nm") is None:
        pytest.skip("nm not available")
    out = subprocess.run(["nm", "-DC", "--defined-only", so_path], capture_output=True, text=True, check=True).stdout
    for name in _declared(os.path.join(INC, "da3cpp", "da3.h"), "DA3_API"):
        assert re.search(r"\bda3::" + name + r"\(", out), f"da3::{name} not exported"


def test_abi_versions_without_gpu(so_path):
    """The version queries touch no device: the reference C ABI reports 4
    (src/da_capi.cpp:71)."""
    from da3cpplib_b200 import _lib

    L = _lib.load()
    assert L.da_capi_abi_version() == 4
    assert L.da3b_abi_version() >= 1


def test_load_missing_file_fails_cleanly(so_path):
    """da_capi_load on a missing GGUF returns NULL (the reference's error convention,
    src/da_capi.cpp:13) before any device work."""
    from da3cpplib_b200 import _lib

    L = _lib.load()
    assert not L.da_capi_load(b"/nonexistent/model.gguf", 1)
    assert not L.da3b_load(b"/nonexistent/model.gguf", 0)
