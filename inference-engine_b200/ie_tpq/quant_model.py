"""Model-level quantization driver -- the API of the reference's ie/quant/model.py.

``quantize_transformer`` keeps the reference's behaviour (fake-quantize every
projection in place, ie/quant/model.py:42-65) so code written against it runs
unchanged, with the tables computed on the GPU.  ``pack_transformer`` is the
real path: it returns each block's projections as packed device shards for one
tensor-parallel rank (column shards for q/k/v/gate/up, row shards for o/down).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .formats import FP8_E4M3, INT4, INT8, FloatFormat, IntegerFormat
from .sharding import Shard, split_heads, split_input_dim, split_output_dim
from .weights import (PER_OUTPUT_CHANNEL, QuantizedWeight, quantize_float, quantize_grouped,
                      quantize_integer, relative_error)

LINEAR_ATTRIBUTES = ("q_proj", "k_proj", "v_proj", "o_proj",
                     "gate_proj", "up_proj", "down_proj")


@dataclass(slots=True)
class QuantizationReport:
    """ie/quant/model.py:15-32."""
    scheme: str
    dense_bytes: int = 0
    stored_bytes: float = 0.0
    errors: list[float] = field(default_factory=list)

    @property
    def compression(self) -> float:
        return self.dense_bytes / self.stored_bytes if self.stored_bytes else 0.0

    @property
    def mean_error(self) -> float:
        return float(np.mean(self.errors)) if self.errors else 0.0

    @property
    def worst_error(self) -> float:
        return float(np.max(self.errors)) if self.errors else 0.0


def quantize_tensor(weight: np.ndarray, fmt: IntegerFormat | FloatFormat,
                    axis: int | None = PER_OUTPUT_CHANNEL) -> QuantizedWeight:
    """ie/quant/model.py:35-39."""
    if isinstance(fmt, IntegerFormat):
        return quantize_integer(weight, fmt, axis)
    return quantize_float(weight, fmt, axis)


def quantize_transformer(model, fmt: IntegerFormat | FloatFormat,
                         axis: int | None = PER_OUTPUT_CHANNEL,
                         include_lm_head: bool = False) -> QuantizationReport:
    """ie/quant/model.py:42-65 -- fake-quantize the model's projections in place."""
    report = QuantizationReport(scheme=f"{fmt.name}/{'tensor' if axis is None else 'channel'}")
    for block in model.blocks:
        for name in LINEAR_ATTRIBUTES:
            original = getattr(block, name)
            packed = quantize_tensor(original, fmt, axis)
            restored = packed.dequantized()
            setattr(block, name, restored)
            report.dense_bytes += packed.dense_bytes
            report.stored_bytes += packed.stored_bytes
            report.errors.append(relative_error(original, restored))
    if include_lm_head:
        packed = quantize_tensor(model.lm_head, fmt, axis)
        report.errors.append(relative_error(model.lm_head, packed.dequantized()))
        report.dense_bytes += packed.dense_bytes
        report.stored_bytes += packed.stored_bytes
        model.lm_head = packed.dequantized()
    return report


def named_format(name: str) -> IntegerFormat | FloatFormat:
    """ie/quant/model.py:68-72."""
    table = {"int8": INT8, "int4": INT4, "fp8": FP8_E4M3}
    if name not in table:
        raise ValueError(f"unknown format {name!r}; expected one of {sorted(table)}")
    return table[name]


def quantize_for_device(weight: np.ndarray, scheme: str,
                        axis: int | None = PER_OUTPUT_CHANNEL) -> QuantizedWeight:
    """``scheme`` in {"int8", "int4", "fp8", "int4-g128"} -> reference-format tables."""
    if scheme == "int4-g128":
        return quantize_grouped(weight)
    return quantize_tensor(weight, named_format(scheme), axis)


def pack_transformer(model, scheme: str, shard: Shard, axis: int | None = PER_OUTPUT_CHANNEL,
                     device=None) -> list[dict]:
    """Per block, this rank's packed projections.

    Keys: q, k, v (head-sharded columns, ie/parallel/tensor_parallel.py:21-23),
    o (row shard, :24), gate_up (gate/up column shards paired for the fused
    SiLU*up epilogue, :50-51) and down (row shard, :52).  Quantization runs on
    the full weight first, as the reference's fake-quant does, so the shard's
    tables are slices of the full tables.
    """
    from .packed import PackedWeight

    cfg = model.config
    blocks = []
    for block in model.blocks:
        q = {name: quantize_for_device(getattr(block, name), scheme, axis)
             for name in LINEAR_ATTRIBUTES}
        packed = {
            "q": split_heads(q["q_proj"], shard, cfg.num_heads, cfg.head_dim).packed(device),
            "k": split_heads(q["k_proj"], shard, cfg.num_kv_heads, cfg.head_dim).packed(device),
            "v": split_heads(q["v_proj"], shard, cfg.num_kv_heads, cfg.head_dim).packed(device),
            "o": split_input_dim(q["o_proj"], shard).packed(device),
            "gate_up": PackedWeight.pair_gate_up(
                split_output_dim(q["gate_proj"], shard).packed(device),
                split_output_dim(q["up_proj"], shard).packed(device)),
            "down": split_input_dim(q["down_proj"], shard).packed(device),
        }
        blocks.append(packed)
    return blocks
