"""Pin the CPU oracle to the reference: every function of oracle/tpq_oracle.py
against the fixtures tests/golden/make_golden.py produced by running the
reference engine itself.  Bit-exact equality throughout (the oracle restates
the same NumPy operations)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import tpq_oracle as o
from tests.hashing import digest


def test_format_constants_match_the_reference(golden):
    assert list(golden["fmt_int"]) == [o.int_signed_max(8), -o.int_signed_max(8),
                                       o.int_unsigned_max(8), o.int_signed_max(4),
                                       -o.int_signed_max(4), o.int_unsigned_max(4)]
    assert list(golden["fmt_float"]) == [o.float_max_value(*o.E4M3), o.float_min_normal(4),
                                         o.float_max_value(*o.E5M2), o.float_min_normal(5)]


def test_round_to_float_format_matches_bitwise(golden):
    x = golden["round_in"]
    assert np.array_equal(o.round_to_float_format(x, *o.E4M3).astype(np.float32),
                          golden["round_e4m3"])
    assert np.array_equal(o.round_to_float_format(x, *o.E5M2).astype(np.float32),
                          golden["round_e5m2"])


@pytest.mark.parametrize("tag,axis", [("k", 0), ("n", 1), ("t", None)])
def test_quantizer_tables_match_bitwise(golden, tag, axis):
    w = golden["w"]
    q = o.quantize_integer(w, 8, True, axis)
    assert np.array_equal(q.codes, golden[f"int8_{tag}_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"int8_{tag}_scale"])
    assert np.array_equal(q.dequantized(), golden[f"int8_{tag}_deq"])
    q = o.quantize_integer(w, 8, False, axis)
    assert np.array_equal(q.codes, golden[f"int8a_{tag}_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"int8a_{tag}_scale"])
    assert np.array_equal(q.zero_point, golden[f"int8a_{tag}_zero"])
    q = o.quantize_integer(w, 4, True, axis)
    assert np.array_equal(q.codes, golden[f"int4_{tag}_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"int4_{tag}_scale"])
    q = o.quantize_float(w, *o.E4M3, axis=axis)
    assert np.array_equal(q.codes, golden[f"fp8_{tag}_codes"])
    assert np.array_equal(q.scale, golden[f"fp8_{tag}_scale"])
    assert np.array_equal(q.dequantized(), golden[f"fp8_{tag}_deq"])


def test_stored_bytes_accounting(golden):
    q = o.quantize_integer(golden["w"], 8, True, 0)
    stored, compression = golden["int8_k_stored_bytes"]
    assert q.stored_bytes == stored
    assert golden["w"].size * 4 / q.stored_bytes == pytest.approx(compression)


def test_group128_restatement_matches_the_reference_on_the_view(golden):
    g = o.quantize_int4_group128(golden["wg"])
    n, k = g.codes.shape
    assert np.array_equal(g.codes.reshape(-1, 128), golden["g128_codes"].astype(np.int32))
    assert np.array_equal(g.scale.reshape(-1, 1), golden["g128_scale"])
    assert np.array_equal(g.zero.reshape(-1, 1), golden["g128_zero"])
    deq_view = golden["g128_deq"].reshape(n, k).T
    assert np.array_equal(g.dequantized(), deq_view)


def test_per_token_fp8_activations(golden):
    q = o.quantize_activations_fp8(golden["act_x"])
    assert np.array_equal(q.codes, golden["act_codes"])
    assert np.array_equal(q.scale, golden["act_scale"])


@pytest.mark.parametrize("name", ["const", "zeros", "onesided", "outlier"])
def test_edge_weights(golden, name):
    w = golden[f"edge_{name}"]
    q = o.quantize_integer(w, 8, True, 0)
    assert np.array_equal(q.codes, golden[f"edge_{name}_int8_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"edge_{name}_int8_scale"])
    q = o.quantize_integer(w, 8, False, None)
    assert np.array_equal(q.codes, golden[f"edge_{name}_int8a_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"edge_{name}_int8a_scale"])
    assert np.array_equal(q.zero_point, golden[f"edge_{name}_int8a_zero"])
    q = o.quantize_float(w, *o.E4M3, axis=0)
    assert np.array_equal(q.codes, golden[f"edge_{name}_fp8_codes"])
    assert np.array_equal(q.scale, golden[f"edge_{name}_fp8_scale"])


def test_shard_splits_match(golden):
    base = golden["shard_base"]
    for world in (1, 2, 3, 4):
        for r in range(world):
            assert np.array_equal(o.split_output_dim(base, r, world), golden[f"col_{world}_{r}"])
            assert np.array_equal(o.split_input_dim(base, r, world), golden[f"row_{world}_{r}"])
    for world in (1, 2, 4):
        for r in range(world):
            assert np.array_equal(o.split_heads(base, r, world, 4, 6), golden[f"heads_{world}_{r}"])


def test_shard_validation_errors():
    with pytest.raises(ValueError):
        o.shard_slice(2, 2, 8)
    with pytest.raises(ValueError):
        o.shard_slice(0, 0, 8)
    with pytest.raises(ValueError):
        o.shard_slice(0, 3, 8)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_sharded_mlp_matches_the_reference(golden, world):
    x = golden["mlp_x"]
    got = o.tp_mlp(x, np.ones(64, np.float32), golden["mlp_gate"], golden["mlp_up"],
                   golden["mlp_down"], world)
    assert np.array_equal(got, golden[f"mlp_out_{world}"])


@pytest.mark.parametrize("world", [1, 2, 4])
def test_row_parallel_all_reduce_matches_the_reference(golden, world):
    w = o.quantize_int4_group128(golden["row_w"]).dequantized()
    got = o.row_parallel_allreduce(golden["row_x"], w, world)
    assert np.array_equal(got, golden[f"row_out_{world}"])


def test_full_size_cpu_case_digests(golden_hashes):
    """hidden 896 / intermediate 4864 / 64 tokens / TP=2 / int8 per-channel."""
    x, norm, gate, up, down = o.config1_inputs()
    deq = {}
    for name, w in (("gate", gate), ("up", up), ("down", down)):
        q = o.quantize_integer(w, 8, True, 0)
        assert digest(q.codes) == golden_hashes[f"config1_{name}_codes"]
        assert digest(q.scale) == golden_hashes[f"config1_{name}_scale"]
        deq[name] = q.dequantized()
    y = o.tp_mlp(x, norm, deq["gate"], deq["up"], deq["down"], 2)
    assert float(np.sum(y.astype(np.float64))) == pytest.approx(
        golden_hashes["config1_out_tp2_sum"], rel=1e-9)
    assert float(np.max(np.abs(y))) == pytest.approx(golden_hashes["config1_out_tp2_absmax"],
                                                     rel=1e-7)
    g = o.quantize_int4_group128(down)
    assert digest(g.codes.reshape(-1, 128)) == golden_hashes["config1_down_g128_codes"]
    assert digest(g.scale.reshape(-1, 1)) == golden_hashes["config1_down_g128_scale"]
    assert digest(g.zero.reshape(-1, 1)) == golden_hashes["config1_down_g128_zero"]
    q = o.quantize_float(down, *o.E4M3, axis=0)
    assert digest(q.codes) == golden_hashes["config1_down_fp8_codes"]
    assert digest(q.scale) == golden_hashes["config1_down_fp8_scale"]
