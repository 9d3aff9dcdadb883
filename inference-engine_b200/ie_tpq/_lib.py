"""ctypes binding of libie_tpq.so (declared in include/ie_tpq.h).

The library is built in-tree next to this file by ``ie_tpq.build``.  There is
no fallback: if the shared object is missing or does not load, every entry
point raises ``RuntimeError`` naming the path and the loader's message.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libie_tpq.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

# status codes (ie_tpq.h)
IE_OK = 0
IE_ERR_INVALID = 1
IE_ERR_CUDA = 2
IE_ERR_TIMEOUT = 3
IE_ERR_UNSUPPORTED = 4

IE_FMT_INT8 = 0
IE_FMT_INT4 = 1
IE_FMT_FP8_E4M3 = 2

IE_AXIS_K = 0
IE_AXIS_N = 1
IE_AXIS_TENSOR = 2
IE_AXIS_GROUP128 = 3

IE_DT_BF16 = 0
IE_DT_F16 = 1
IE_DT_F32 = 2
IE_DT_I32 = 3
IE_DT_U8 = 4

IE_EPI_BIAS = 1
IE_EPI_RESIDUAL = 2
IE_EPI_SILU_MUL = 4
IE_EPI_RMS_NORM = 8
IE_ACT_NONE, IE_ACT_FP8_TOKEN = 0, 1
# all-reduce protocols (the algo argument of ie_qlinear_allreduce / ie_allreduce)
IE_AR_AUTO, IE_AR_ONESHOT, IE_AR_TWOSHOT, IE_AR_NVLS = 0, 1, 2, 3

IE_COMM_HANDLE_BYTES = 64
IE_QLINEAR_NOALLOC_SCRATCH_BYTES = 8 << 20

# every symbol include/ie_tpq.h declares
EXPORTED = (
    "ie_version", "ie_last_error", "ie_quantize_integer", "ie_quantize_float",
    "ie_round_to_float_format", "ie_pack_weight", "ie_dequantize",
    "ie_qlinear_workspace_size", "ie_qlinear", "ie_qlinear_noalloc", "ie_kernel_status",
    "ie_rms_norm", "ie_rope_kv",
    "ie_reduce_partials", "ie_comm_create",
    "ie_comm_export", "ie_comm_open", "ie_comm_destroy", "ie_comm_set_timeout",
    "ie_comm_check", "ie_qlinear_allreduce", "ie_allreduce", "ie_allreduce_resolve",
)


class QWeight(ctypes.Structure):
    _fields_ = [
        ("format", ctypes.c_int32),
        ("axis", ctypes.c_int32),
        ("k", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("codes", ctypes.c_void_p),
        ("scale", ctypes.c_void_p),
        ("zero", ctypes.c_void_p),
        ("int4_symmetric", ctypes.c_int32),
        ("gate_up", ctypes.c_int32),
    ]


class QLinearArgs(ctypes.Structure):
    _fields_ = [
        ("w", QWeight),
        ("m", ctypes.c_int64),
        ("act_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("ldx", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("ldo", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("ldr", ctypes.c_int64),
        ("epilogue", ctypes.c_int32),
        ("algo", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
        ("act_quant", ctypes.c_int32),
    ]


_lib: ctypes.CDLL | None = None
_load_error: str | None = None

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64


def _declare(lib: ctypes.CDLL) -> None:
    sig = {
        "ie_version": (ctypes.c_int, []),
        "ie_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
        "ie_quantize_integer": (ctypes.c_int, [_P, _I64, _I64, _I32, _I32, _I32, _P, _P, _P, _P]),
        "ie_quantize_float": (ctypes.c_int, [_P, _I64, _I64, _I32, _I32, _I32, _I32, _P, _P, _P]),
        "ie_round_to_float_format": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _I32, _P]),
        "ie_pack_weight": (ctypes.c_int, [_I32, _I32, _I32, _I64, _I64, _P, _P, _P, _P, _P, _P,
                                          _P, _P]),
        "ie_dequantize": (ctypes.c_int, [ctypes.POINTER(QWeight), _I32, _I32, _P, _P]),
        "ie_qlinear_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(QLinearArgs)]),
        "ie_qlinear": (ctypes.c_int, [ctypes.POINTER(QLinearArgs), _P]),
        "ie_qlinear_noalloc": (ctypes.c_int, [ctypes.POINTER(QLinearArgs), _P]),
        "ie_kernel_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _I32]),
        "ie_rms_norm": (ctypes.c_int, [_P, _I64, _I32, _P, _P, _I64, _I32, _I64, _I64,
                                       ctypes.c_float, _P]),
        "ie_rope_kv": (ctypes.c_int, [_P, _I64, _I32, _I64, _I32, _I32, _I32, _P, _P, _P, _I64,
                                      _I32, _P, _P, _P, _I64, _P, _P]),
        "ie_reduce_partials": (ctypes.c_int, [ctypes.POINTER(_P), _I32, _P, _I64, _I32, _P]),
        "ie_comm_create": (ctypes.c_int, [_I32, _I32, _I32, ctypes.c_size_t,
                                          ctypes.POINTER(_P)]),
        "ie_comm_export": (ctypes.c_int, [_P, _P]),
        "ie_comm_open": (ctypes.c_int, [_P, _P]),
        "ie_comm_destroy": (ctypes.c_int, [_P]),
        "ie_comm_set_timeout": (ctypes.c_int, [_P, ctypes.c_uint64]),
        "ie_comm_check": (ctypes.c_int, [_P]),
        "ie_qlinear_allreduce": (ctypes.c_int, [_P, ctypes.POINTER(QLinearArgs), _I32, _P]),
        "ie_allreduce": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _P]),
        "ie_allreduce_resolve": (ctypes.c_int, [_I32, _I64, _I64, _I32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> ctypes.CDLL:
    """The loaded library; raises RuntimeError (no fallback) when it is unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    path = os.environ.get("IE_TPQ_LIB", str(LIB_PATH))
    if not Path(path).exists():
        raise RuntimeError(f"{path} is missing: build it with `python -m ie_tpq.build` "
                           "(the quantized TP path has no CPU fallback)")
    try:
        handle = ctypes.CDLL(path)
    except OSError as exc:
        _load_error = str(exc)
        raise RuntimeError(f"cannot load {path}: {exc}") from exc
    _declare(handle)
    _lib = handle
    return handle


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().ie_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


class TimeoutError_(RuntimeError):
    """A bounded wait for a peer rank ran out (IE_ERR_TIMEOUT)."""


def check(code: int, what: str = "") -> None:
    """Map a status code to the reference's exception types.

    IE_ERR_INVALID -> ValueError (the reference raises ValueError for bad
    ranks, uneven splits and unknown formats: ie/parallel/sharding.py:13-21,
    ie/quant/model.py:70-71); everything else -> RuntimeError.
    """
    if code == IE_OK:
        return
    msg = last_error()
    prefix = f"{what}: " if what else ""
    if code == IE_ERR_INVALID:
        raise ValueError(prefix + msg)
    if code == IE_ERR_TIMEOUT:
        raise TimeoutError_(prefix + msg)
    raise RuntimeError(prefix + f"[status {code}] " + msg)


def stream_ptr(stream=None) -> int | None:
    """Raw cudaStream_t of a torch stream (the current one when None)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None
