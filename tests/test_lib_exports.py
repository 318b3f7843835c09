"""The C-ABI library loads and exports every entry point include/pir2b.h
declares (no compute calls: this runs without a GPU)."""

import ctypes
import os
import re

import pytest

from pir2_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pir2b.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pir2b_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert {"pir2b_quant_rows", "pir2b_gemm", "pir2b_norm_quant_rows", "pir2b_pack_nvfp4"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) <= set(_lib.SIGNATURES)


def test_version_and_error_string_without_gpu():
    lib = _lib.lib()
    assert lib.pir2b_version() >= 100
    assert isinstance(lib.pir2b_last_error(), bytes)


def test_argument_errors_are_reported_without_touching_the_device():
    lib = _lib.lib()
    status = lib.pir2b_quant_rows(None, 0, None, 0, None, None, 0, 3, 1, 8, None, None, None)
    assert status == _lib.EINVAL
    assert b"bits" in lib.pir2b_last_error()
    status = lib.pir2b_gemm(None, None, None, None, None, 0, None, None, 0, 8, 1, 12, 128, None, 12, 12, -1, None)
    assert status == _lib.EINVAL
    with pytest.raises(ValueError, match="npad"):
        _lib.check(status, "pir2b_gemm")
