"""Tensor-parallel sharding -- the API of the reference's ie/parallel/sharding.py.

Same names, arguments and errors (``ValueError`` for a bad rank, world size
or uneven split, ie/parallel/sharding.py:13-21).  The split functions are
index arithmetic and work on every weight form:

  * a dense NumPy array or torch tensor -> a view, exactly as the reference;
  * a ``QuantizedWeight`` (host tables)  -> the same slice of codes, scales and
    zero points, so ``shard(q).dequantized() == shard(q.dequantized())``;
  * a ``PackedWeight`` (device)           -> the packed rows / K range.

``ColumnParallelLinear`` / ``RowParallelLinear`` run the quantized shard on
the GPU.  ``RowParallelLinear.forward(x_shard)`` returns the rank's partial as
the reference does; ``forward(x_shard, reduce=comm)`` returns the reduced sum
with the all-reduce fused into the GEMM epilogue.  ``all_reduce`` on a list
keeps the reference's rank-order f32 summation.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import numpy as np

from . import _lib
from .device import dtype_code, require_cuda
from .packed import PackedWeight
from .weights import QuantizedWeight


@dataclass(frozen=True, slots=True)
class Shard:
    """ie/parallel/sharding.py:8-23."""
    rank: int
    world_size: int

    def __post_init__(self):
        if self.world_size < 1:
            raise ValueError("world_size must be at least 1")
        if not 0 <= self.rank < self.world_size:
            raise ValueError(f"rank {self.rank} outside world of {self.world_size}")

    def slice_of(self, length: int) -> slice:
        if length % self.world_size:
            raise ValueError(f"{length} does not divide evenly across {self.world_size} ranks")
        width = length // self.world_size
        return slice(self.rank * width, (self.rank + 1) * width)


def _shape(weight):
    if isinstance(weight, QuantizedWeight):
        return tuple(weight.original_shape)
    if isinstance(weight, PackedWeight):
        return (weight.k, weight.n)
    return tuple(weight.shape)


def _slice_quantized_cols(q: QuantizedWeight, sl: slice) -> QuantizedWeight:
    k, n = q.original_shape
    width = sl.stop - sl.start
    if q.group_size:
        return replace(q, codes=q.codes[sl], scale=q.scale[sl],
                       zero_point=q.zero_point[sl], original_shape=(k, width))
    scale = q.scale[:, sl] if q.scale.shape[1] == n and n > 1 else q.scale
    zero = None
    if q.zero_point is not None:
        zero = q.zero_point[:, sl] if q.zero_point.shape[1] == n and n > 1 else q.zero_point
    return replace(q, codes=q.codes[:, sl], scale=scale, zero_point=zero,
                   original_shape=(k, width))


def _slice_quantized_rows(q: QuantizedWeight, sl: slice) -> QuantizedWeight:
    k, n = q.original_shape
    height = sl.stop - sl.start
    if q.group_size:
        g = q.group_size
        if sl.start % g or sl.stop % g:
            raise ValueError(f"a K shard [{sl.start}, {sl.stop}) splits a group of {g}")
        gs = slice(sl.start // g, sl.stop // g)
        return replace(q, codes=q.codes[:, sl], scale=q.scale[:, gs],
                       zero_point=q.zero_point[:, gs], original_shape=(height, n))
    scale = q.scale[sl, :] if q.scale.shape[0] == k and k > 1 else q.scale
    zero = None
    if q.zero_point is not None:
        zero = q.zero_point[sl, :] if q.zero_point.shape[0] == k and k > 1 else q.zero_point
    return replace(q, codes=q.codes[sl, :], scale=scale, zero_point=zero,
                   original_shape=(height, n))


def split_output_dim(weight, shard: Shard):
    """ie/parallel/sharding.py:26-27 -- column shard ``W[:, slice]``."""
    sl = shard.slice_of(_shape(weight)[1])
    if isinstance(weight, QuantizedWeight):
        return _slice_quantized_cols(weight, sl)
    if isinstance(weight, PackedWeight):
        return weight.slice_rows(sl.start, sl.stop)
    return weight[:, sl]


def split_input_dim(weight, shard: Shard):
    """ie/parallel/sharding.py:30-31 -- row shard ``W[slice, :]``."""
    sl = shard.slice_of(_shape(weight)[0])
    if isinstance(weight, QuantizedWeight):
        return _slice_quantized_rows(weight, sl)
    if isinstance(weight, PackedWeight):
        return weight.slice_k(sl.start, sl.stop)
    return weight[sl, :]


def split_heads(weight, shard: Shard, num_heads: int, head_dim: int):
    """ie/parallel/sharding.py:34-37 -- head-contiguous column shard.

    A head block of ``head_dim`` columns is contiguous, so a rank's heads are
    the contiguous column range ``[r*H/w*hd, (r+1)*H/w*hd)``."""
    per_rank = shard.slice_of(num_heads)
    cols = slice(per_rank.start * head_dim, per_rank.stop * head_dim)
    if _shape(weight)[1] != num_heads * head_dim:
        raise ValueError(f"weight has {_shape(weight)[1]} columns, expected "
                         f"{num_heads} heads x {head_dim}")
    if isinstance(weight, QuantizedWeight):
        return _slice_quantized_cols(weight, cols)
    if isinstance(weight, PackedWeight):
        return weight.slice_rows(cols.start, cols.stop)
    reshaped = weight.reshape(weight.shape[0], num_heads, head_dim)
    return reshaped[:, per_rank, :].reshape(weight.shape[0], -1)


def all_reduce(partials):
    """ie/parallel/sharding.py:40-44 -- ``partials[0] + partials[1] + ...`` in rank order.

    NumPy partials keep the reference's exact semantics: a copy of the first,
    then ``+=`` of the others in rank order, in the partials' own dtype, on the
    host (the reference's expert-parallel combine, ie/parallel/expert_parallel.py:57,
    sums NumPy lists through this function).  CUDA tensors are summed on the GPU
    by ``ie_reduce_partials`` (f32 arithmetic, rank order) and stay on the device."""
    if not partials:
        raise ValueError("all_reduce needs at least one partial")
    if isinstance(partials[0], np.ndarray) or np.isscalar(partials[0]):
        total = np.array(partials[0], copy=True)
        for part in partials[1:]:
            total += part
        return total
    torch = require_cuda()
    dev = partials[0].device if partials[0].is_cuda else torch.device("cuda")
    ts = [p.to(dev).contiguous() for p in partials]
    shape = ts[0].shape
    for t in ts[1:]:
        if t.shape != shape or t.dtype != ts[0].dtype:
            raise ValueError("all partials must share shape and dtype")
    out = torch.empty_like(ts[0])
    arr = (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    _lib.check(_lib.lib().ie_reduce_partials(arr, len(ts), out.data_ptr(), out.numel(),
                                             dtype_code(out.dtype), _lib.stream_ptr()),
               "all_reduce")
    return out


def all_gather(partials, axis: int = -1):
    """ie/parallel/sharding.py:47-48 -- concatenation (a copy; no arithmetic)."""
    if partials and not isinstance(partials[0], np.ndarray):
        import torch

        return torch.cat(list(partials), dim=axis)
    return np.concatenate(partials, axis=axis)


def _packed(weight, device=None) -> PackedWeight:
    if isinstance(weight, PackedWeight):
        return weight
    if isinstance(weight, QuantizedWeight):
        return PackedWeight.from_quantized(weight, device=device)
    raise TypeError("the device linear layers take a QuantizedWeight or PackedWeight; "
                    f"got {type(weight).__name__} (quantize it with ie_tpq.weights first)")


def _as_device(x, dtype=None):
    torch = require_cuda()
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda(), True
    return (x if x.is_cuda else x.cuda()), False


class ColumnParallelLinear:
    """ie/parallel/sharding.py:51-57 on the GPU: ``x @ W[:, this rank's columns]``."""

    def __init__(self, weight, shard: Shard, device=None) -> None:
        self.shard = shard
        self.weight = _packed(split_output_dim(weight, shard), device)

    def forward(self, x, *, bias=None):
        from .linear import qlinear

        xt, was_numpy = _as_device(x)
        y = qlinear(xt, self.weight, bias=bias, silu_mul=False)
        return y.cpu().numpy() if was_numpy else y


class RowParallelLinear:
    """ie/parallel/sharding.py:60-66 on the GPU: the rank's partial
    ``x_shard @ W[this rank's rows, :]``; with ``reduce=comm`` the partials of
    all ranks are summed inside the kernel and the reduced output returned."""

    def __init__(self, weight, shard: Shard, device=None) -> None:
        self.shard = shard
        self.weight = _packed(split_input_dim(weight, shard), device)

    def forward(self, x_shard, *, reduce=None, residual=None, bias=None):
        from .linear import qlinear

        xt, was_numpy = _as_device(x_shard)
        res = None
        if residual is not None:
            res, _ = _as_device(residual)
            res = res.to(xt.dtype)
        y = qlinear(xt, self.weight, residual=res, bias=bias, comm=reduce)
        return y.cpu().numpy() if was_numpy else y
