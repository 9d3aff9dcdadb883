"""Host-side logic of the ie_tpq mirror that needs no GPU: shard arithmetic,
validation errors (ValueError, as the reference raises), format descriptions
and slicing of quantized tables.  Modelled on the reference's
tests/test_tensor_parallel.py:25-56,118-122 and tests/test_quantization.py:32-42."""
from __future__ import annotations

import numpy as np
import pytest

from ie_tpq import formats as F
from ie_tpq.quant_model import LINEAR_ATTRIBUTES, named_format
from ie_tpq.sharding import Shard, all_gather, split_heads, split_input_dim, split_output_dim
from ie_tpq.tensor_parallel import kv_heads_per_rank
from ie_tpq.weights import QuantizedWeight
from oracle import tpq_oracle as o


def test_shard_rejects_an_out_of_range_rank():
    with pytest.raises(ValueError):
        Shard(rank=2, world_size=2)
    with pytest.raises(ValueError):
        Shard(rank=0, world_size=0)
    with pytest.raises(ValueError):
        Shard(rank=-1, world_size=2)


def test_shard_rejects_an_uneven_split():
    with pytest.raises(ValueError):
        Shard(rank=0, world_size=3).slice_of(8)


def test_column_shards_concatenate_back_to_the_whole_weight():
    weight = np.arange(24, dtype=np.float32).reshape(4, 6)
    pieces = [split_output_dim(weight, Shard(r, 3)) for r in range(3)]
    assert np.array_equal(all_gather(pieces, axis=-1), weight)


def test_row_shards_stack_back_to_the_whole_weight():
    weight = np.arange(24, dtype=np.float32).reshape(6, 4)
    pieces = [split_input_dim(weight, Shard(r, 3)) for r in range(3)]
    assert np.array_equal(np.concatenate(pieces, axis=0), weight)


def test_head_sharding_keeps_each_head_contiguous():
    num_heads, head_dim = 4, 3
    weight = np.arange(2 * num_heads * head_dim, dtype=np.float32).reshape(2, num_heads * head_dim)
    left = split_heads(weight, Shard(0, 2), num_heads, head_dim)
    right = split_heads(weight, Shard(1, 2), num_heads, head_dim)
    assert left.shape == (2, 2 * head_dim)
    assert np.array_equal(all_gather([left, right], axis=-1), weight)


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_splits_equal_the_oracle(world):
    base = np.arange(12 * 24, dtype=np.float32).reshape(12, 24)
    for r in range(world):
        assert np.array_equal(split_output_dim(base, Shard(r, world)),
                              o.split_output_dim(base, r, world))
        assert np.array_equal(split_input_dim(base, Shard(r, world)),
                              o.split_input_dim(base, r, world))


def _qw(codes, scale, zero=None, bits=8, group=None, shape=None):
    return QuantizedWeight(codes=codes, scale=scale, zero_point=zero, format_name="t", bits=bits,
                           original_shape=shape or codes.shape, group_size=group)


@pytest.mark.parametrize("axis", [0, 1, None])
@pytest.mark.parametrize("world", [1, 2, 4])
def test_sharding_quantized_tables_commutes_with_dequantize(axis, world):
    """shard(q).dequantized() == shard(q.dequantized()) for every axis."""
    w = o.seeded_weight(64, 32, seed=3)
    q = o.quantize_integer(w, 8, True, axis)
    qw = _qw(q.codes, q.scale)
    full = q.dequantized()
    for r in range(world):
        sh = Shard(r, world)
        for split, osplit in ((split_output_dim, o.split_output_dim),
                              (split_input_dim, o.split_input_dim)):
            part = split(qw, sh)
            deq = o.OracleQuantized(part.codes, part.scale, None, 8).dequantized()
            assert np.array_equal(deq, osplit(full, r, world))


@pytest.mark.parametrize("world", [1, 2])
def test_sharding_group128_tables(world):
    w = o.seeded_weight(256, 64, seed=4)
    g = o.quantize_int4_group128(w)
    qw = _qw(g.codes, g.scale, g.zero, bits=4, group=128, shape=(256, 64))
    full = g.dequantized()
    for r in range(world):
        sh = Shard(r, world)
        col = split_output_dim(qw, sh)
        assert col.original_shape == (256, 64 // world)
        assert np.array_equal(o.OracleGroup128(col.codes, col.scale, col.zero_point).dequantized(),
                              o.split_output_dim(full, r, world))
        row = split_input_dim(qw, sh)
        assert row.original_shape == (256 // world, 64)
        assert np.array_equal(o.OracleGroup128(row.codes, row.scale, row.zero_point).dequantized(),
                              o.split_input_dim(full, r, world))


def test_group128_row_shard_must_not_split_a_group():
    w = o.seeded_weight(256, 8, seed=5)
    g = o.quantize_int4_group128(w)
    qw = _qw(g.codes, g.scale, g.zero, bits=4, group=128, shape=(256, 8))
    with pytest.raises(ValueError):
        split_input_dim(qw, Shard(0, 4))   # 64-row shards cut the 128-groups


def test_format_descriptions_match_the_reference():
    assert F.INT8.signed_max == 127 and F.INT8.signed_min == -127
    assert F.INT4.signed_max == 7 and F.INT8.unsigned_max == 255
    assert F.FP8_E4M3.bits == 8
    assert F.FP8_E4M3.max_value == pytest.approx(448.0)
    assert F.FP8_E5M2.max_value == pytest.approx(57344.0)
    assert F.INT8_ASYM.name == "int8-asym" and F.FP8_E4M3.name == "fp8-e4m3"


def test_named_format_rejects_an_unknown_name():
    assert named_format("int8") is F.INT8
    with pytest.raises(ValueError):
        named_format("int3")
    assert LINEAR_ATTRIBUTES == ("q_proj", "k_proj", "v_proj", "o_proj",
                                 "gate_proj", "up_proj", "down_proj")


def test_format_ids_reject_formats_without_a_device_layout():
    assert F.format_id(F.INT8) == 0 and F.format_id(F.INT4) == 1 and F.format_id(F.FP8_E4M3) == 2
    with pytest.raises(ValueError):
        F.format_id(F.INT8_ASYM)
    with pytest.raises(ValueError):
        F.format_id(F.FP8_E5M2)


class _Cfg:
    num_kv_heads = 2


def test_kv_cache_shrinks_proportionally_with_world_size():
    assert kv_heads_per_rank(_Cfg, 1) == 2
    assert kv_heads_per_rank(_Cfg, 2) == 1
    with pytest.raises(ValueError):
        kv_heads_per_rank(_Cfg, 4)


def test_compression_accounting_matches_the_reference():
    w = o.seeded_weight(256, 256, seed=6)
    q8 = o.quantize_integer(w, 8, True, 0)
    q4 = o.quantize_integer(w, 4, True, 0)
    assert _qw(q8.codes, q8.scale).compression == pytest.approx(4.0, rel=0.05)
    assert _qw(q4.codes, q4.scale, bits=4).compression == pytest.approx(8.0, rel=0.05)


def test_all_reduce_on_numpy_lists_is_the_references_host_sum():
    """ie/parallel/sharding.py:40-44: a copy of the first partial, then += in
    rank order, in the partials' dtype, with no GPU (expert parallelism sums
    NumPy lists through it, ie/parallel/expert_parallel.py:57)."""
    from ie_tpq.sharding import all_reduce
    from oracle import tpq_oracle as o

    parts = [o.seeded_activations(7, 33, seed=s) for s in range(4)]
    got = all_reduce(parts)
    assert got.dtype == np.float32 and np.array_equal(got, o.all_reduce(parts))
    assert got is not parts[0] and not np.shares_memory(got, parts[0])
    ints = [np.arange(6, dtype=np.int64) * (r + 1) for r in range(3)]
    assert all_reduce(ints).dtype == np.int64
    assert np.array_equal(all_reduce(ints), np.arange(6) * 6)
    f64 = [np.full(3, 0.1, np.float64)] * 3
    assert all_reduce(f64).dtype == np.float64
    with pytest.raises(ValueError):
        all_reduce([])
