"""Weight quantizer -- the API of the reference's ie/quant/weights.py.

``quantize_integer`` / ``quantize_float`` keep the reference's signatures,
axis convention (``axis`` is the KEPT dimension; ``PER_OUTPUT_CHANNEL = 0``
keeps K of a ``[K, N]`` weight, ie/quant/weights.py:9-10,45-48) and return a
``QuantizedWeight`` of host arrays with the same fields, but the tables are
computed on the GPU by ``ie_quantize_integer`` / ``ie_quantize_float``, which
reproduce the reference's f32 arithmetic bit for bit.  ``dequantized()`` runs
on the GPU as well.

``quantize_grouped`` adds the int4 asymmetric group-128 scheme: the
reference's own ``quantize_integer`` applied to the ``[N*K/128, 128]`` view of
``W.T`` (one scale and zero point per output column and 128-long K group).

``.packed()`` turns any of them into the device layout the kernels stream
(``PackedWeight``, ie_tpq.packed).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib
from .device import require_cuda
from .formats import FloatFormat, IntegerFormat

PER_TENSOR = None
PER_OUTPUT_CHANNEL = 0
GROUP_SIZE = 128


@dataclass(slots=True)
class QuantizedWeight:
    """ie/quant/weights.py:13-42; ``group_size`` marks the group-128 layout
    (codes ``[N, K]``, scale/zero ``[N, K/128]`` for a ``[K, N]`` weight)."""
    codes: np.ndarray
    scale: np.ndarray
    zero_point: np.ndarray | None
    format_name: str
    bits: int
    original_shape: tuple[int, ...]
    group_size: int | None = None

    def dequantized(self) -> np.ndarray:
        """ie/quant/weights.py:22-26, computed on the GPU in f32."""
        torch = require_cuda()
        codes = torch.from_numpy(np.ascontiguousarray(self.codes)).cuda().to(torch.float32)
        if self.group_size:
            n, k = self.codes.shape
            codes = codes.reshape(n * k // self.group_size, self.group_size)
            scale = torch.from_numpy(self.scale.reshape(-1, 1)).cuda()
            zero = torch.from_numpy(self.zero_point.reshape(-1, 1)).cuda()
            out = (codes - zero) * scale
            return out.reshape(n, k).t().contiguous().cpu().numpy()
        if self.zero_point is not None:
            codes = codes - torch.from_numpy(self.zero_point).cuda()
        out = codes * torch.from_numpy(self.scale).cuda()
        return out.to(torch.float32).cpu().numpy()

    @property
    def stored_bytes(self) -> float:
        """ie/quant/weights.py:28-34 (the reference's accounting)."""
        payload = self.codes.size * self.bits / 8
        overhead = self.scale.size * 4
        if self.zero_point is not None:
            overhead += self.zero_point.size * 4
        return payload + overhead

    @property
    def dense_bytes(self) -> int:
        return int(np.prod(self.original_shape)) * 4

    @property
    def compression(self) -> float:
        return self.dense_bytes / self.stored_bytes

    def packed(self, device=None, gate_up_with=None):
        """Device layout for the kernels (see ie_tpq.packed.PackedWeight)."""
        from .packed import PackedWeight

        return PackedWeight.from_quantized(self, device=device)


def _to_rows(weight: np.ndarray, axis: int | None):
    """Move the kept axis first and flatten the rest: returns (2-D view, kernel axis)."""
    if axis is None:
        return weight.reshape(1, -1), -1
    if not -weight.ndim <= axis < weight.ndim:
        raise ValueError(f"axis {axis} out of range for a {weight.ndim}-D weight")
    axis = axis % weight.ndim
    if weight.ndim == 2:
        return weight, axis
    moved = np.moveaxis(weight, axis, 0)
    return moved.reshape(moved.shape[0], -1), 0


def _keepdims(shape, axis):
    if axis is None:
        return tuple(1 for _ in shape)
    axis = axis % len(shape)
    return tuple(s if d == axis else 1 for d, s in enumerate(shape))


def _from_rows(codes2d: np.ndarray, weight: np.ndarray, axis):
    if axis is None or weight.ndim == 2:
        return codes2d.reshape(weight.shape)
    axis = axis % weight.ndim
    moved_shape = (weight.shape[axis],) + tuple(s for d, s in enumerate(weight.shape) if d != axis)
    return np.moveaxis(codes2d.reshape(moved_shape), 0, axis)


def quantize_integer(weight: np.ndarray, fmt: IntegerFormat,
                     axis: int | None = PER_OUTPUT_CHANNEL) -> QuantizedWeight:
    """ie/quant/weights.py:51-70 on the GPU (bit-exact tables)."""
    torch = require_cuda()
    weight = np.asarray(weight, dtype=np.float32)
    if weight.size == 0:
        raise ValueError("cannot quantize an empty weight")
    rows2d, kaxis = _to_rows(np.ascontiguousarray(weight), axis)
    rows, cols = rows2d.shape
    w = torch.from_numpy(np.ascontiguousarray(rows2d)).cuda()
    nscale = rows if kaxis == 0 else (cols if kaxis == 1 else 1)
    codes = torch.empty((rows, cols), dtype=torch.int32, device=w.device)
    scale = torch.empty(nscale, dtype=torch.float32, device=w.device)
    zero = None if fmt.symmetric else torch.empty(nscale, dtype=torch.float32, device=w.device)
    _lib.check(_lib.lib().ie_quantize_integer(
        w.data_ptr(), rows, cols, fmt.bits, int(fmt.symmetric), kaxis, codes.data_ptr(),
        scale.data_ptr(), zero.data_ptr() if zero is not None else None, _lib.stream_ptr()),
        "quantize_integer")
    keep = _keepdims(weight.shape, axis)
    return QuantizedWeight(
        codes=_from_rows(codes.cpu().numpy(), weight, axis),
        scale=scale.cpu().numpy().reshape(keep),
        zero_point=None if zero is None else zero.cpu().numpy().reshape(keep),
        format_name=f"{fmt.name}/{'tensor' if axis is None else 'channel'}",
        bits=fmt.bits, original_shape=weight.shape)


def quantize_float(weight: np.ndarray, fmt: FloatFormat,
                   axis: int | None = PER_OUTPUT_CHANNEL) -> QuantizedWeight:
    """ie/quant/weights.py:73-81 on the GPU (bit-exact tables, f32 codes)."""
    torch = require_cuda()
    weight = np.asarray(weight, dtype=np.float32)
    if weight.size == 0:
        raise ValueError("cannot quantize an empty weight")
    rows2d, kaxis = _to_rows(np.ascontiguousarray(weight), axis)
    rows, cols = rows2d.shape
    w = torch.from_numpy(np.ascontiguousarray(rows2d)).cuda()
    nscale = rows if kaxis == 0 else (cols if kaxis == 1 else 1)
    codes = torch.empty((rows, cols), dtype=torch.float32, device=w.device)
    scale = torch.empty(nscale, dtype=torch.float32, device=w.device)
    _lib.check(_lib.lib().ie_quantize_float(
        w.data_ptr(), rows, cols, fmt.exponent_bits, fmt.mantissa_bits,
        int(fmt.reserves_infinity), kaxis, codes.data_ptr(), scale.data_ptr(),
        _lib.stream_ptr()), "quantize_float")
    return QuantizedWeight(
        codes=_from_rows(codes.cpu().numpy(), weight, axis),
        scale=scale.cpu().numpy().reshape(_keepdims(weight.shape, axis)),
        zero_point=None,
        format_name=f"{fmt.name}/{'tensor' if axis is None else 'channel'}",
        bits=fmt.bits, original_shape=weight.shape)


def quantize_grouped(weight: np.ndarray, fmt: IntegerFormat | None = None,
                     group_size: int = GROUP_SIZE) -> QuantizedWeight:
    """int4 asymmetric group-128 of a ``[K, N]`` weight: the reference's
    ``quantize_integer(W.T.reshape(N*K/128, 128), IntegerFormat(4, False), axis=0)``."""
    fmt = fmt or IntegerFormat(4, symmetric=False)
    if fmt.bits != 4 or fmt.symmetric or group_size != GROUP_SIZE:
        raise ValueError("grouped quantization is int4 asymmetric with groups of 128")
    weight = np.asarray(weight, dtype=np.float32)
    if weight.ndim != 2:
        raise ValueError("grouped quantization takes a 2-D [K, N] weight")
    k, n = weight.shape
    if k % group_size:
        raise ValueError(f"K={k} is not a multiple of the group size {group_size}")
    view = np.ascontiguousarray(weight.T).reshape(n * k // group_size, group_size)
    q = quantize_integer(view, fmt, axis=0)
    return QuantizedWeight(codes=q.codes.reshape(n, k),
                           scale=q.scale.reshape(n, k // group_size),
                           zero_point=q.zero_point.reshape(n, k // group_size),
                           format_name=f"{fmt.name}/group{group_size}", bits=4,
                           original_shape=(k, n), group_size=group_size)


def relative_error(original: np.ndarray, reconstructed: np.ndarray) -> float:
    """ie/quant/weights.py:84-88 (a host-side metric, not part of the compute path)."""
    denominator = np.linalg.norm(original)
    if denominator == 0:
        return 0.0
    return float(np.linalg.norm(original - reconstructed) / denominator)


def max_absolute_error(original: np.ndarray, reconstructed: np.ndarray) -> float:
    """ie/quant/weights.py:91-92."""
    return float(np.max(np.abs(original - reconstructed)))
