"""The C-ABI library loads without a GPU, exports every entry point that
include/ie_tpq.h declares, and rejects bad arguments with IE_ERR_INVALID
before touching CUDA (so these run on the CPU-only build machine)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ie_tpq import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "ie_tpq.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:int|size_t)\s+(ie_\w+)\s*\(", text, flags=re.M))


def test_header_declarations_match_the_binding_table():
    assert declared_symbols() == set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.ie_version() == 3


def test_invalid_arguments_are_rejected_before_any_cuda_call():
    lib = _lib.lib()
    assert lib.ie_qlinear(None, None) == _lib.IE_ERR_INVALID
    a = _lib.QLinearArgs()
    a.w.format = 7
    a.w.codes = 16
    a.w.scale = 16
    a.w.k, a.w.n = 64, 64
    assert lib.ie_qlinear(ctypes.byref(a), None) == _lib.IE_ERR_INVALID
    assert "unknown format" in _lib.last_error()
    a.w.format = _lib.IE_FMT_INT4
    a.w.axis = _lib.IE_AXIS_GROUP128
    a.w.k = 96
    assert lib.ie_qlinear(ctypes.byref(a), None) == _lib.IE_ERR_INVALID
    h = ctypes.c_void_p()
    assert lib.ie_comm_create(0, 9, 0, 1024, ctypes.byref(h)) == _lib.IE_ERR_INVALID
    assert lib.ie_comm_create(2, 2, 0, 1024, ctypes.byref(h)) == _lib.IE_ERR_INVALID
    assert lib.ie_reduce_partials(None, 1, None, 4, 2, None) == _lib.IE_ERR_INVALID


def test_status_codes_map_to_the_reference_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.IE_ERR_INVALID)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.IE_ERR_CUDA)
    with pytest.raises(_lib.TimeoutError_):
        _lib.check(_lib.IE_ERR_TIMEOUT)
