"""CPU oracle for the tensor-parallel quantized linear path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the ``ie_tpq`` package and
``libie_tpq.so``) imports, calls or links this module.  It is imported only by
``tests/``, by ``__graft_entry__.smoke()`` (as the checker) and by ``bench.py``'s
CPU-baseline leg and ``--impl reference`` arm (as the timed CPU implementation).

It is a plain-NumPy restatement of the reference engine's arithmetic for this
path (kuluruvineeth/inference-engine, pure Python + NumPy).  Every function
names the reference file:line it restates.  Parity of this restatement is
PINNED: ``tests/test_oracle_golden.py`` checks it bit-for-bit against the
fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
importing and running the reference itself.

Two pieces have no counterpart in the reference's defaults and are restated
with the reference's own functions on reshaped views:
  * int4 asymmetric group-128 (``quantize_int4_group128``): the reference's
    ``quantize_integer`` applied to a ``[N*K/128, 128]`` view of ``W.T``;
  * per-token fp8 activation scales (``quantize_activations_fp8``): the
    reference's ``quantize_float`` applied row-wise to ``x [M, K]``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# ---------------------------------------------------------------------------
# Sharding (ie/parallel/sharding.py)
# ---------------------------------------------------------------------------


def shard_slice(rank: int, world_size: int, length: int) -> slice:
    """ie/parallel/sharding.py:13-23 -- validity checks then an even split."""
    if world_size < 1:
        raise ValueError("world_size must be at least 1")
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    if length % world_size:
        raise ValueError(f"{length} does not divide evenly across {world_size} ranks")
    width = length // world_size
    return slice(rank * width, (rank + 1) * width)


def split_output_dim(weight: np.ndarray, rank: int, world: int) -> np.ndarray:
    """ie/parallel/sharding.py:26-27 -- column shard W[:, slice]."""
    return weight[:, shard_slice(rank, world, weight.shape[1])]


def split_input_dim(weight: np.ndarray, rank: int, world: int) -> np.ndarray:
    """ie/parallel/sharding.py:30-31 -- row shard W[slice, :]."""
    return weight[shard_slice(rank, world, weight.shape[0]), :]


def split_heads(weight: np.ndarray, rank: int, world: int, num_heads: int,
                head_dim: int) -> np.ndarray:
    """ie/parallel/sharding.py:34-37 -- head-contiguous column shard."""
    per_rank = shard_slice(rank, world, num_heads)
    reshaped = weight.reshape(weight.shape[0], num_heads, head_dim)
    return reshaped[:, per_rank, :].reshape(weight.shape[0], -1)


def all_reduce(partials: list[np.ndarray]) -> np.ndarray:
    """ie/parallel/sharding.py:40-44 -- copy of rank 0, then += in rank order."""
    total = partials[0].copy()
    for part in partials[1:]:
        total += part
    return total


def all_gather(partials: list[np.ndarray], axis: int = -1) -> np.ndarray:
    """ie/parallel/sharding.py:47-48."""
    return np.concatenate(partials, axis=axis)


# ---------------------------------------------------------------------------
# Formats (ie/quant/formats.py)
# ---------------------------------------------------------------------------


def int_signed_max(bits: int) -> int:
    """ie/quant/formats.py:20-22 -- (2^bits)/2 - 1; signed_min is its negation (:24-26)."""
    return (1 << bits) // 2 - 1


def int_unsigned_max(bits: int) -> int:
    """ie/quant/formats.py:28-30."""
    return (1 << bits) - 1


def float_max_value(exponent_bits: int, mantissa_bits: int, reserves_infinity: bool) -> float:
    """ie/quant/formats.py:50-59."""
    bias = (1 << (exponent_bits - 1)) - 1
    if reserves_infinity:
        largest = (1 << exponent_bits) - 2 - bias
        mscale = 2.0 - 2.0 ** (-mantissa_bits)
    else:
        largest = (1 << exponent_bits) - 1 - bias
        mscale = 2.0 - 2.0 ** (1 - mantissa_bits)
    return float(2.0 ** largest * mscale)


def float_min_normal(exponent_bits: int) -> float:
    """ie/quant/formats.py:61-63."""
    bias = (1 << (exponent_bits - 1)) - 1
    return float(2.0 ** (1 - bias))


E4M3 = (4, 3, False)   # ie/quant/formats.py:70  (max 448)
E5M2 = (5, 2, True)    # ie/quant/formats.py:71  (max 57344)


def round_to_float_format(x: np.ndarray, exponent_bits: int = 4, mantissa_bits: int = 3,
                          reserves_infinity: bool = False) -> np.ndarray:
    """ie/quant/formats.py:74-79.

    clip to +-max, frexp (mantissa in [0.5, 1)), round(m * 2^mb) / 2^mb with
    NumPy's half-to-even, ldexp, clip again, flush |v| < min_normal * 2^-mb to 0.
    Because the frexp mantissa is in [0.5, 1), only mb-1 fraction bits survive.
    """
    max_value = float_max_value(exponent_bits, mantissa_bits, reserves_infinity)
    min_normal = float_min_normal(exponent_bits)
    mantissa, exponent = np.frexp(np.clip(x, -max_value, max_value))
    quantum = 1 << mantissa_bits
    out = np.ldexp(np.round(mantissa * quantum) / quantum, exponent)
    out = np.clip(out, -max_value, max_value)
    return np.where(np.abs(out) < min_normal * 2.0 ** -mantissa_bits, 0.0, out)


# ---------------------------------------------------------------------------
# Weight quantizer (ie/quant/weights.py)
# ---------------------------------------------------------------------------


@dataclass
class OracleQuantized:
    """ie/quant/weights.py:13-20 -- codes, scale, optional zero point."""
    codes: np.ndarray
    scale: np.ndarray
    zero_point: np.ndarray | None
    bits: int

    def dequantized(self) -> np.ndarray:
        """ie/quant/weights.py:22-26."""
        codes = self.codes.astype(np.float32)
        if self.zero_point is not None:
            codes = codes - self.zero_point
        return (codes * self.scale).astype(np.float32)

    @property
    def stored_bytes(self) -> float:
        """ie/quant/weights.py:28-34."""
        payload = self.codes.size * self.bits / 8
        overhead = self.scale.size * 4
        if self.zero_point is not None:
            overhead += self.zero_point.size * 4
        return payload + overhead


def reduce_axes(ndim: int, axis: int | None) -> tuple[int, ...]:
    """ie/quant/weights.py:45-48 -- ``axis`` is the KEPT dimension."""
    if axis is None:
        return tuple(range(ndim))
    return tuple(d for d in range(ndim) if d != axis)


def quantize_integer(weight: np.ndarray, bits: int, symmetric: bool = True,
                     axis: int | None = 0) -> OracleQuantized:
    """ie/quant/weights.py:51-70."""
    axes = reduce_axes(weight.ndim, axis)
    if symmetric:
        qmax = int_signed_max(bits)
        peak = np.max(np.abs(weight), axis=axes, keepdims=True)
        scale = np.where(peak == 0, 1.0, peak / qmax).astype(np.float32)
        codes = np.clip(np.round(weight / scale), -qmax, qmax)
        zero_point = None
    else:
        umax = int_unsigned_max(bits)
        low = np.min(weight, axis=axes, keepdims=True)
        high = np.max(weight, axis=axes, keepdims=True)
        span = np.where(high - low == 0, 1.0, high - low)
        scale = (span / umax).astype(np.float32)
        zero_point = np.round(-low / scale).astype(np.float32)
        codes = np.clip(np.round(weight / scale + zero_point), 0, umax)
    return OracleQuantized(codes.astype(np.int32), scale, zero_point, bits)


def quantize_float(weight: np.ndarray, exponent_bits: int = 4, mantissa_bits: int = 3,
                   reserves_infinity: bool = False, axis: int | None = 0) -> OracleQuantized:
    """ie/quant/weights.py:73-81 -- scale = max|w| / fmt.max_value, codes stay f32."""
    max_value = float_max_value(exponent_bits, mantissa_bits, reserves_infinity)
    axes = reduce_axes(weight.ndim, axis)
    peak = np.max(np.abs(weight), axis=axes, keepdims=True)
    scale = np.where(peak == 0, 1.0, peak / max_value).astype(np.float32)
    codes = round_to_float_format(weight / scale, exponent_bits, mantissa_bits,
                                  reserves_infinity)
    return OracleQuantized(codes.astype(np.float32), scale, None,
                           1 + exponent_bits + mantissa_bits)


def relative_error(original: np.ndarray, reconstructed: np.ndarray) -> float:
    """ie/quant/weights.py:84-88."""
    denominator = np.linalg.norm(original)
    if denominator == 0:
        return 0.0
    return float(np.linalg.norm(original - reconstructed) / denominator)


# ---------------------------------------------------------------------------
# Restatements with no default in the reference (built from its own functions)
# ---------------------------------------------------------------------------

GROUP = 128


@dataclass
class OracleGroup128:
    """int4 asymmetric group-128 tables for a ``[K, N]`` weight.

    codes ``[N, K]`` int32 in [0, 15]; scale and zero ``[N, K/128]`` f32, exactly
    as ie/quant/weights.py:60-66 computes them on the ``[N*K/128, 128]`` view.
    """
    codes: np.ndarray
    scale: np.ndarray
    zero: np.ndarray

    def dequantized(self) -> np.ndarray:
        """``[K, N]`` f32 -- ie/quant/weights.py:22-26 on the view, transposed back."""
        n, k = self.codes.shape
        view = self.codes.reshape(n * k // GROUP, GROUP).astype(np.float32)
        deq = (view - self.zero.reshape(-1, 1)) * self.scale.reshape(-1, 1)
        return deq.astype(np.float32).reshape(n, k).T.copy()


def quantize_int4_group128(weight: np.ndarray) -> OracleGroup128:
    """Reference ``quantize_integer(W.T.reshape(N*K/128, 128), IntegerFormat(4, False), axis=0)``."""
    k, n = weight.shape
    if k % GROUP:
        raise ValueError(f"K={k} is not a multiple of the group size {GROUP}")
    view = np.ascontiguousarray(weight.T).reshape(n * k // GROUP, GROUP)
    q = quantize_integer(view, 4, symmetric=False, axis=0)
    return OracleGroup128(q.codes.reshape(n, k), q.scale.reshape(n, k // GROUP),
                          q.zero_point.reshape(n, k // GROUP))


def quantize_activations_fp8(x: np.ndarray) -> OracleQuantized:
    """Per-token e4m3 activation scales: reference ``quantize_float(x, FP8_E4M3, axis=0)``."""
    return quantize_float(x, *E4M3, axis=0)


# ---------------------------------------------------------------------------
# Functional layers and the sharded MLP/linear (ie/layers/functional.py,
# ie/parallel/tensor_parallel.py)
# ---------------------------------------------------------------------------


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """ie/layers/functional.py:6-8."""
    scale = np.sqrt(np.mean(np.square(x, dtype=np.float32), axis=-1, keepdims=True) + eps)
    return (x / scale) * weight


def silu(x: np.ndarray) -> np.ndarray:
    """ie/layers/functional.py:11-12."""
    return x / (1.0 + np.exp(-x))


def sharded_mlp_partial(x: np.ndarray, norm: np.ndarray, gate: np.ndarray, up: np.ndarray,
                        down: np.ndarray, rank: int, world: int,
                        eps: float = 1e-6) -> np.ndarray:
    """ie/parallel/tensor_parallel.py:46-56 -- one rank's partial of the SwiGLU MLP."""
    normed = rms_norm(x, norm, eps)
    g = normed @ split_output_dim(gate, rank, world)
    u = normed @ split_output_dim(up, rank, world)
    return (silu(g) * u) @ split_input_dim(down, rank, world)


def tp_mlp(x: np.ndarray, norm: np.ndarray, gate: np.ndarray, up: np.ndarray,
           down: np.ndarray, world: int, eps: float = 1e-6) -> np.ndarray:
    """ie/parallel/tensor_parallel.py:72-73 -- ``x + all_reduce(partials)`` for the MLP."""
    partials = [sharded_mlp_partial(x, norm, gate, up, down, r, world, eps)
                for r in range(world)]
    return x + all_reduce(partials)


def column_parallel(x: np.ndarray, weight: np.ndarray, rank: int, world: int) -> np.ndarray:
    """ie/parallel/sharding.py:51-57."""
    return x @ split_output_dim(weight, rank, world)


def row_parallel(x_shard: np.ndarray, weight: np.ndarray, rank: int, world: int) -> np.ndarray:
    """ie/parallel/sharding.py:60-66 -- the partial; the caller reduces it."""
    return x_shard @ split_input_dim(weight, rank, world)


def row_parallel_allreduce(x: np.ndarray, weight: np.ndarray, world: int) -> np.ndarray:
    """Every rank's row-parallel partial, reduced by ``all_reduce`` in rank order."""
    partials = []
    for r in range(world):
        x_shard = x[:, shard_slice(r, world, x.shape[1])]
        partials.append(row_parallel(x_shard, weight, r, world))
    return all_reduce(partials)


# ---------------------------------------------------------------------------
# Seeded synthetic inputs shared by tests, smoke() and bench.py
# ---------------------------------------------------------------------------


def seeded_weight(k: int, n: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    """N(0, std) f32 weight in the reference's ``[K_in, N_out]`` layout."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((k, n)) * std).astype(np.float32)


def seeded_activations(m: int, k: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.standard_normal((m, k)).astype(np.float32)


def config1_inputs(seed: int = 0):
    """The CPU-runnable MLP case: hidden 896, intermediate 4864, tokens 64, N(0, 0.02) weights."""
    rng = np.random.default_rng(seed)
    hidden, inter, tokens = 896, 4864, 64
    gate = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)
    up = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)
    down = (rng.standard_normal((inter, hidden)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, hidden)).astype(np.float32)
    norm = np.ones(hidden, dtype=np.float32)
    return x, norm, gate, up, down
