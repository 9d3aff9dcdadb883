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
    assert lib.ie_version() == 4


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


def test_allreduce_protocol_resolution():
    """IE_AR_AUTO keeps one-shot for decode-sized outputs and below world 4 (two-shot
    sends as many bytes at world 2); two-shot needs one output tile per rank."""
    from ie_tpq.comm import AR_AUTO, AR_NVLS, AR_ONESHOT, AR_TWOSHOT, resolve_algo

    # decode: 16 tokens x 4096 columns, 32 tiles
    for world in (1, 2, 4, 8):
        assert resolve_algo(world, 32, 16 * 4096) == AR_ONESHOT
    # prefill: 2048 tokens x 4096 columns
    assert resolve_algo(2, 256, 2048 * 4096) == AR_ONESHOT
    assert resolve_algo(4, 256, 2048 * 4096) == AR_TWOSHOT
    assert resolve_algo(8, 256, 2048 * 4096) == AR_TWOSHOT
    # the crossover at world 8: 2.5 MB saved = 21 bytes per element
    assert resolve_algo(8, 64, 119_000) == AR_ONESHOT
    assert resolve_algo(8, 64, 120_000) == AR_TWOSHOT
    # explicit choices; two-shot with fewer tiles than ranks runs one-shot
    assert resolve_algo(2, 32, 64, AR_TWOSHOT) == AR_TWOSHOT
    assert resolve_algo(8, 4, 1 << 24, AR_TWOSHOT) == AR_ONESHOT
    assert resolve_algo(8, 4096, 1 << 24, AR_ONESHOT) == AR_ONESHOT
    with pytest.raises(ValueError):
        resolve_algo(8, 64, 1 << 20, AR_NVLS)
    with pytest.raises(ValueError):
        resolve_algo(9, 64, 1 << 20, AR_AUTO)
    lib = _lib.lib()
    assert lib.ie_allreduce(None, None, None, 4, 2, 0, None) == _lib.IE_ERR_INVALID


def test_status_codes_map_to_the_reference_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.IE_ERR_INVALID)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.IE_ERR_CUDA)
    with pytest.raises(_lib.TimeoutError_):
        _lib.check(_lib.IE_ERR_TIMEOUT)
