"""CPU checks of the C ABI: the library loads, exports every symbol include/w8a8.h declares,
and rejects bad arguments without touching a GPU."""
from __future__ import annotations

import ctypes as C
import re

import pytest
import torch

from conftest import ROOT
from romanaccio_b200 import _lib


def header_functions() -> list[str]:
    text = (ROOT / "include" / "w8a8.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w8a8_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    names = header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_status_strings():
    lib = _lib.load()
    for code in range(0, -12, -1):
        s = lib.w8a8_status_to_string(code).decode()
        assert s and s != "unknown status"
    assert lib.w8a8_status_to_string(5).decode() == "unknown status"
    assert b"sm_100a" in lib.w8a8_version()


def test_null_arguments_are_rejected():
    lib = _lib.load()
    assert lib.w8a8_ctx_create(0, None) == _lib.ERR_INVALID_ARG
    h = C.c_void_p()
    assert lib.w8a8_linear_create(None, None, C.byref(h)) == _lib.ERR_INVALID_ARG
    assert lib.w8a8_ctx_check(None) == _lib.ERR_INVALID_ARG
    assert lib.w8a8_linear_forward(None, None, 0, 1, 0, 0, None, 0, None, None) == _lib.ERR_INVALID_ARG
    assert lib.w8a8_topk_merge(None, None, None, 1, 1, 1, 1, 1, 1, None, None, None, None) == \
        _lib.ERR_INVALID_ARG
    assert lib.w8a8_linear_reserve(None, 64, 40, None) == _lib.ERR_INVALID_ARG
    assert "NULL" in lib.w8a8_last_error().decode()
    lib.w8a8_linear_destroy(None)  # NULL-safe like es_*_free
    lib.w8a8_ctx_destroy(None)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_ctx_create_reports_missing_device():
    lib = _lib.load()
    h = C.c_void_p()
    st = lib.w8a8_ctx_create(0, C.byref(h))
    assert st in (_lib.ERR_NOT_INITIALIZED, _lib.ERR_CUDA)
    assert not h.value
