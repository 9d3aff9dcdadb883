"""Weight formats -- the API of the reference's ie/quant/formats.py.

``IntegerFormat`` / ``FloatFormat`` and the five named constants are plain
descriptions (ie/quant/formats.py:8-71), kept with the same fields and
properties so code written against the reference reads the same.
``round_to_float_format`` (ie/quant/formats.py:74-79) runs on the GPU through
``ie_round_to_float_format``; it accepts NumPy arrays (returned as NumPy) or
CUDA tensors (returned as CUDA tensors).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib


@dataclass(frozen=True, slots=True)
class IntegerFormat:
    """ie/quant/formats.py:8-31 -- symmetric range is +-(2^(b-1)-1)."""
    bits: int
    symmetric: bool = True

    @property
    def name(self) -> str:
        return f"int{self.bits}{'' if self.symmetric else '-asym'}"

    @property
    def num_levels(self) -> int:
        return 1 << self.bits

    @property
    def signed_max(self) -> int:
        return (self.num_levels // 2) - 1

    @property
    def signed_min(self) -> int:
        return -self.signed_max

    @property
    def unsigned_max(self) -> int:
        return self.num_levels - 1


@dataclass(frozen=True, slots=True)
class FloatFormat:
    """ie/quant/formats.py:34-64."""
    exponent_bits: int
    mantissa_bits: int
    reserves_infinity: bool = True

    @property
    def name(self) -> str:
        return (f"fp{1 + self.exponent_bits + self.mantissa_bits}"
                f"-e{self.exponent_bits}m{self.mantissa_bits}")

    @property
    def bits(self) -> int:
        return 1 + self.exponent_bits + self.mantissa_bits

    @property
    def exponent_bias(self) -> int:
        return (1 << (self.exponent_bits - 1)) - 1

    @property
    def max_value(self) -> float:
        if self.reserves_infinity:
            largest_exponent = (1 << self.exponent_bits) - 2 - self.exponent_bias
            mantissa_scale = 2.0 - 2.0 ** (-self.mantissa_bits)
        else:
            largest_exponent = (1 << self.exponent_bits) - 1 - self.exponent_bias
            mantissa_scale = 2.0 - 2.0 ** (1 - self.mantissa_bits)
        return float(2.0 ** largest_exponent * mantissa_scale)

    @property
    def min_normal(self) -> float:
        return float(2.0 ** (1 - self.exponent_bias))


INT8 = IntegerFormat(bits=8)
INT4 = IntegerFormat(bits=4)
INT8_ASYM = IntegerFormat(bits=8, symmetric=False)
FP8_E4M3 = FloatFormat(exponent_bits=4, mantissa_bits=3, reserves_infinity=False)
FP8_E5M2 = FloatFormat(exponent_bits=5, mantissa_bits=2)


def round_to_float_format(x, fmt: FloatFormat):
    """GPU restatement of ie/quant/formats.py:74-79 (bit-exact)."""
    import torch

    from .device import to_device_f32

    t, was_numpy, shape = to_device_f32(x)
    out = torch.empty_like(t)
    _lib.check(_lib.lib().ie_round_to_float_format(
        t.data_ptr(), out.data_ptr(), t.numel(), fmt.exponent_bits, fmt.mantissa_bits,
        int(fmt.reserves_infinity), _lib.stream_ptr()), "round_to_float_format")
    if was_numpy:
        return out.cpu().numpy().reshape(shape)
    return out.reshape(shape)


def format_id(fmt) -> int:
    """The C-ABI format code of a reference format object."""
    if isinstance(fmt, IntegerFormat):
        if fmt.bits == 8 and fmt.symmetric:
            return _lib.IE_FMT_INT8
        if fmt.bits == 4:
            return _lib.IE_FMT_INT4
        raise ValueError(f"{fmt.name} has no packed device layout (int8 symmetric, int4 only)")
    if isinstance(fmt, FloatFormat):
        if (fmt.exponent_bits, fmt.mantissa_bits, fmt.reserves_infinity) == (4, 3, False):
            return _lib.IE_FMT_FP8_E4M3
        raise ValueError(f"{fmt.name} has no packed device layout (fp8-e4m3 only)")
    raise ValueError(f"unknown format {fmt!r}")


__all__ = ["IntegerFormat", "FloatFormat", "INT8", "INT4", "INT8_ASYM", "FP8_E4M3", "FP8_E5M2",
           "round_to_float_format", "format_id"]
