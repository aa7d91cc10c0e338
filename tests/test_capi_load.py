"""CPU checks of the C-ABI library: it loads and exports every declared symbol.

No compute call is made here (there is no GPU on this side).
"""
import ctypes
import glob
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

LIB = os.path.join(PKG, "libuocr_q8.so")


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(uocr_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def built():
    if not os.path.exists(LIB):
        subprocess.run(["make", "-s", "-C", PKG], check=True)
    return LIB


def test_header_declares_functions():
    assert len(declared_functions()) >= 25


def test_library_exports_every_declared_symbol(built):
    lib = ctypes.CDLL(built)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_header(built):
    import uocr_q8._lib as L
    assert sorted(L.SIGNATURES) == declared_functions()
    lib = L.load()
    assert lib.uocr_abi_version() == 1
    assert lib.uocr_status_name(4) == b"Shape"
    assert lib.uocr_status_name(7) == b"Numerical"


def test_no_cpu_fallback_exports(built):
    # the product library never links the oracle
    out = subprocess.run(["nm", "-D", built], capture_output=True, text=True).stdout
    assert "q8o_" not in out


def test_null_arguments_rejected_without_device(built):
    import uocr_q8._lib as L
    lib = L.load()
    h = ctypes.c_void_p()
    assert lib.uocr_q8_from_parts(None, 1, 1, None, 1, None, 1, ctypes.byref(h)) == 11
    assert lib.uocr_ctx_create(0, 0, ctypes.byref(h)) == 6  # scratch 0 -> Resource
