"""GPU quantizer parity: the tables ie_quantize_integer / ie_quantize_float
compute equal the reference's bit for bit (golden fixtures from the reference
itself, and the pinned oracle at sizes with no fixture)."""
from __future__ import annotations

import numpy as np
import pytest

from ie_tpq import formats as F
from ie_tpq import weights as W
from oracle import tpq_oracle as o
from tests.hashing import digest

pytestmark = pytest.mark.gpu

AXES = [("k", 0), ("n", 1), ("t", None)]


def test_round_to_float_format_is_bitwise(golden):
    x = golden["round_in"]
    assert np.array_equal(F.round_to_float_format(x, F.FP8_E4M3), golden["round_e4m3"])
    assert np.array_equal(F.round_to_float_format(x, F.FP8_E5M2), golden["round_e5m2"])


def test_round_to_float_format_is_idempotent_and_clamps():
    x = np.array([1.0, 1.0625, 1.125, 2.5, -3.75], dtype=np.float32)
    once = F.round_to_float_format(x, F.FP8_E4M3)
    assert np.array_equal(once, F.round_to_float_format(once, F.FP8_E4M3))
    out = F.round_to_float_format(np.array([1e6, -1e6], dtype=np.float32), F.FP8_E4M3)
    assert np.all(np.abs(out) <= F.FP8_E4M3.max_value)


@pytest.mark.parametrize("tag,axis", AXES)
def test_tables_match_the_reference_fixtures(golden, tag, axis):
    w = golden["w"]
    q = W.quantize_integer(w, F.INT8, axis)
    assert np.array_equal(q.codes, golden[f"int8_{tag}_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"int8_{tag}_scale"])
    assert np.array_equal(q.dequantized(), golden[f"int8_{tag}_deq"])
    q = W.quantize_integer(w, F.INT8_ASYM, axis)
    assert np.array_equal(q.codes, golden[f"int8a_{tag}_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"int8a_{tag}_scale"])
    assert np.array_equal(q.zero_point, golden[f"int8a_{tag}_zero"])
    q = W.quantize_integer(w, F.INT4, axis)
    assert np.array_equal(q.codes, golden[f"int4_{tag}_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"int4_{tag}_scale"])
    q = W.quantize_float(w, F.FP8_E4M3, axis)
    assert np.array_equal(q.codes, golden[f"fp8_{tag}_codes"])
    assert np.array_equal(q.scale, golden[f"fp8_{tag}_scale"])
    assert np.array_equal(q.dequantized(), golden[f"fp8_{tag}_deq"])


def test_group128_tables_match_the_reference_fixture(golden):
    q = W.quantize_grouped(golden["wg"])
    assert np.array_equal(q.codes.reshape(-1, 128), golden["g128_codes"].astype(np.int32))
    assert np.array_equal(q.scale.reshape(-1, 1), golden["g128_scale"])
    assert np.array_equal(q.zero_point.reshape(-1, 1), golden["g128_zero"])
    n, k = q.codes.shape
    assert np.array_equal(q.dequantized(), golden["g128_deq"].reshape(n, k).T)


def test_per_token_activation_scales(golden):
    q = W.quantize_float(golden["act_x"], F.FP8_E4M3, 0)
    assert np.array_equal(q.codes, golden["act_codes"])
    assert np.array_equal(q.scale, golden["act_scale"])


@pytest.mark.parametrize("name", ["const", "zeros", "onesided", "outlier"])
def test_edge_weights(golden, name):
    w = golden[f"edge_{name}"]
    q = W.quantize_integer(w, F.INT8)
    assert np.array_equal(q.codes, golden[f"edge_{name}_int8_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"edge_{name}_int8_scale"])
    q = W.quantize_integer(w, F.INT8_ASYM, None)
    assert np.array_equal(q.codes, golden[f"edge_{name}_int8a_codes"].astype(np.int32))
    assert np.array_equal(q.scale, golden[f"edge_{name}_int8a_scale"])
    assert np.array_equal(q.zero_point, golden[f"edge_{name}_int8a_zero"])
    q = W.quantize_float(w, F.FP8_E4M3)
    assert np.array_equal(q.codes, golden[f"edge_{name}_fp8_codes"])
    assert np.array_equal(q.scale, golden[f"edge_{name}_fp8_scale"])


def test_all_zero_weight_does_not_divide_by_zero():
    w = np.zeros((4, 4), dtype=np.float32)
    assert np.allclose(W.quantize_integer(w, F.INT8).dequantized(), 0.0)
    assert np.allclose(W.quantize_float(w, F.FP8_E4M3).dequantized(), 0.0)


@pytest.mark.parametrize("shape", [(37, 53), (1, 300), (300, 1), (512, 2048)])
@pytest.mark.parametrize("axis", [0, 1, None])
def test_odd_and_large_shapes_match_the_oracle(shape, axis):
    w = o.seeded_weight(*shape, seed=sum(shape), std=0.5)
    for bits, sym in ((8, True), (8, False), (4, True), (4, False)):
        got = W.quantize_integer(w, F.IntegerFormat(bits, sym), axis)
        want = o.quantize_integer(w, bits, sym, axis)
        assert np.array_equal(got.codes, want.codes)
        assert np.array_equal(got.scale, want.scale)
        if not sym:
            assert np.array_equal(got.zero_point, want.zero_point)
    got = W.quantize_float(w, F.FP8_E4M3, axis)
    want = o.quantize_float(w, *o.E4M3, axis=axis)
    assert np.array_equal(got.codes, want.codes)
    assert np.array_equal(got.scale, want.scale)


def test_three_dimensional_weight_keeps_the_axis():
    w = np.random.default_rng(9).standard_normal((4, 6, 8)).astype(np.float32)
    q = W.quantize_integer(w, F.INT8, axis=1)
    assert q.scale.shape == (1, 6, 1)
    peak = np.max(np.abs(w), axis=(0, 2), keepdims=True)
    assert np.array_equal(q.scale, (peak / 127).astype(np.float32))
    assert np.array_equal(q.codes, np.clip(np.round(w / q.scale), -127, 127).astype(np.int32))


def test_full_size_cpu_case_tables(golden_hashes):
    _, _, gate, up, down = o.config1_inputs()
    for name, w in (("gate", gate), ("up", up), ("down", down)):
        q = W.quantize_integer(w, F.INT8)
        assert digest(q.codes) == golden_hashes[f"config1_{name}_codes"]
        assert digest(q.scale) == golden_hashes[f"config1_{name}_scale"]
    q = W.quantize_grouped(down)
    assert digest(q.codes.reshape(-1, 128)) == golden_hashes["config1_down_g128_codes"]
    assert digest(q.scale.reshape(-1, 1)) == golden_hashes["config1_down_g128_scale"]
    assert digest(q.zero_point.reshape(-1, 1)) == golden_hashes["config1_down_g128_zero"]
    q = W.quantize_float(down, F.FP8_E4M3)
    assert digest(q.codes) == golden_hashes["config1_down_fp8_codes"]
    assert digest(q.scale) == golden_hashes["config1_down_fp8_scale"]
