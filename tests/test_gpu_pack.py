"""Packing parity: the device layouts decode back to the reference's codes bit
for bit, the f32 scale tables are copied exactly, the group-128 f16 tables are
the documented casts, and the dequantized device weight equals the
reference's ``dequantized()`` (exactly where the tables are f32)."""
from __future__ import annotations

import numpy as np
import pytest

from ie_tpq import _lib
from ie_tpq import formats as F
from ie_tpq import weights as W
from ie_tpq.packed import PackedWeight
from ie_tpq.sharding import Shard, split_input_dim, split_output_dim
from oracle import tpq_oracle as o
from tests.unpack import e4m3_to_f32, nearest_e4m3, unpack_int4

pytestmark = pytest.mark.gpu

K, N = 256, 96


@pytest.mark.parametrize("axis", [0, 1, None])
def test_int8_roundtrip(axis):
    w = o.seeded_weight(K, N, seed=1)
    q = W.quantize_integer(w, F.INT8, axis)
    p = q.packed()
    assert p.fmt == _lib.IE_FMT_INT8
    assert np.array_equal(p.codes.cpu().numpy().view(np.int8).astype(np.int32), q.codes.T)
    assert np.array_equal(p.scale.cpu().numpy(), q.scale.reshape(-1))
    assert np.array_equal(p.dequantize().cpu().numpy(), o.quantize_integer(w, 8, True, axis)
                          .dequantized())


@pytest.mark.parametrize("axis", [0, 1, None])
def test_int4_symmetric_roundtrip(axis):
    w = o.seeded_weight(K, N, seed=2)
    q = W.quantize_integer(w, F.INT4, axis)
    p = q.packed()
    assert p.int4_symmetric
    assert np.array_equal(unpack_int4(p.codes.cpu().numpy(), K) - 8, q.codes.T)
    assert np.array_equal(p.dequantize().cpu().numpy(), q.dequantized())


def test_int4_group128_roundtrip():
    w = o.seeded_weight(K, N, seed=3)
    q = W.quantize_grouped(w)
    p = q.packed()
    assert p.axis == _lib.IE_AXIS_GROUP128
    assert np.array_equal(unpack_int4(p.codes.cpu().numpy(), K), q.codes)
    assert np.array_equal(p.scale.cpu().numpy(), q.scale.astype(np.float16).T)
    assert np.array_equal(p.zero.cpu().numpy(), q.zero_point.astype(np.float16).T)
    # dequant with the f16 tables: (q - z16) * s16 in f32
    s16 = q.scale.astype(np.float16).astype(np.float32)
    z16 = q.zero_point.astype(np.float16).astype(np.float32)
    view = q.codes.reshape(-1, 128).astype(np.float32)
    want = ((view - z16.reshape(-1, 1)) * s16.reshape(-1, 1)).reshape(N, K).T
    assert np.array_equal(p.dequantize().cpu().numpy(), want)
    ref = o.quantize_int4_group128(w).dequantized()
    assert np.allclose(p.dequantize().cpu().numpy(), ref, rtol=2e-3, atol=1e-6)


@pytest.mark.parametrize("axis", [0, 1])
def test_fp8_roundtrip_counts_unrepresentable_codes(axis):
    w = o.seeded_weight(896, 512, seed=4)
    q = W.quantize_float(w, F.FP8_E4M3, axis)
    p = q.packed()
    stored = e4m3_to_f32(p.codes.cpu().numpy()).T
    nearest = nearest_e4m3(q.codes)
    assert np.array_equal(stored, nearest)
    assert p.unrepresentable == int(np.count_nonzero(nearest != q.codes))
    exact = nearest == q.codes
    deq = p.dequantize().cpu().numpy()
    assert np.array_equal(deq[exact], q.dequantized()[exact])


def test_packed_shards_equal_shards_of_the_packed_weight():
    w = o.seeded_weight(512, 128, seed=5)
    for q in (W.quantize_integer(w, F.INT8), W.quantize_grouped(w),
              W.quantize_float(w, F.FP8_E4M3, 1)):
        full = q.packed()
        for world in (2, 4):
            for r in range(world):
                sh = Shard(r, world)
                a = split_output_dim(q, sh).packed().dequantize().cpu().numpy()
                b = split_output_dim(full, sh).dequantize().cpu().numpy()
                assert np.array_equal(a, b)
                a = split_input_dim(q, sh).packed().dequantize().cpu().numpy()
                b = split_input_dim(full, sh).dequantize().cpu().numpy()
                assert np.array_equal(a, b)


def test_gate_up_pairs_interleave_rows():
    g = W.quantize_integer(o.seeded_weight(128, 64, seed=6), F.INT8).packed()
    u = W.quantize_integer(o.seeded_weight(128, 64, seed=7), F.INT8).packed()
    pair = PackedWeight.pair_gate_up(g, u)
    assert pair.gate_up and pair.n == 128 and pair.out_features == 64
    d = pair.dequantize("nk").cpu().numpy()
    assert np.array_equal(d[0::2], g.dequantize("nk").cpu().numpy())
    assert np.array_equal(d[1::2], u.dequantize("nk").cpu().numpy())


def test_group_tables_that_f16_cannot_hold_are_rejected():
    w = np.full((128, 4), 5000.0, dtype=np.float32)
    w[0] = 5000.001   # tiny span on a large offset -> a huge zero point
    q = W.quantize_grouped(w)
    with pytest.raises(ValueError):
        q.packed()
