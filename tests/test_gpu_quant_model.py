"""The model-level quantization driver on the device: ``quantize_tensor``,
``quantize_transformer`` and ``pack_transformer`` (ie/quant/model.py:35-72),
mirroring the reference's tests/test_quantization.py:120-149 on its own test
configuration, plus the packed shards against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ie_tpq import formats as F
from ie_tpq.packed import PackedWeight
from ie_tpq.quant_model import (LINEAR_ATTRIBUTES, named_format, pack_transformer,
                                quantize_tensor, quantize_transformer)
from ie_tpq.sharding import Shard
from oracle import model_oracle as mo
from oracle import tpq_oracle as o

pytestmark = pytest.mark.gpu

CONFIG = mo.Config(vocab_size=128, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                   head_dim=16, intermediate_size=128)


def test_quantize_tensor_dispatches_on_the_format():
    w = o.seeded_weight(64, 96, seed=3)
    qi = quantize_tensor(w, F.INT8)
    assert qi.bits == 8 and qi.zero_point is None and qi.scale.shape == (64, 1)
    assert np.array_equal(qi.dequantized(), o.quantize_integer(w, 8, True, 0).dequantized())
    qf = quantize_tensor(w, F.FP8_E4M3)
    assert qf.codes.dtype == np.float32
    assert np.array_equal(qf.dequantized(), o.quantize_float(w, *o.E4M3, axis=0).dequantized())
    qa = quantize_tensor(w, F.INT8_ASYM, axis=1)
    want = o.quantize_integer(w, 8, False, 1)
    assert np.array_equal(qa.zero_point, want.zero_point)


def test_quantizing_the_model_reports_compression_and_error():
    """tests/test_quantization.py:128-133."""
    model = mo.Model(CONFIG, seed=1)
    report = quantize_transformer(model, F.INT8)
    assert report.compression > 3.5
    assert report.mean_error < 0.02
    assert report.worst_error < 0.05
    assert len(report.errors) == CONFIG.num_layers * len(LINEAR_ATTRIBUTES)


def test_quantize_transformer_fake_quantizes_in_place_like_the_reference():
    model = mo.Model(CONFIG, seed=1)
    originals = {n: getattr(model.blocks[1], n).copy() for n in LINEAR_ATTRIBUTES}
    lm = model.lm_head.copy()
    quantize_transformer(model, F.INT4)
    for n, w in originals.items():
        assert np.array_equal(getattr(model.blocks[1], n),
                              o.quantize_integer(w, 4, True, 0).dequantized()), n
    assert np.array_equal(model.lm_head, lm)   # include_lm_head defaults to False
    report = quantize_transformer(model, F.INT8, include_lm_head=True)
    assert not np.array_equal(model.lm_head, lm)
    assert len(report.errors) == CONFIG.num_layers * len(LINEAR_ATTRIBUTES) + 1


def test_lower_precision_has_larger_error():
    a, b = mo.Model(CONFIG, seed=2), mo.Model(CONFIG, seed=2)
    assert quantize_transformer(a, F.INT8).mean_error < quantize_transformer(b, F.INT4).mean_error


def test_named_format_rejects_an_unknown_name():
    """tests/test_quantization.py:122-125."""
    assert named_format("int8") is F.INT8
    with pytest.raises(ValueError):
        named_format("int3")


@pytest.mark.parametrize("scheme,world", [("int8", 1), ("int8", 2), ("int4-g128", 2),
                                          ("fp8", 2)])
def test_pack_transformer_shards_match_the_oracle(scheme, world):
    cfg = mo.Config(vocab_size=128, hidden_size=256, num_layers=1, num_heads=4,
                    num_kv_heads=2, head_dim=64, intermediate_size=512)
    model = mo.Model(cfg, seed=7)
    blk = model.blocks[0]
    x = o.seeded_activations(5, cfg.hidden_size, seed=8)
    for r in range(world):
        packed = pack_transformer(model, scheme, Shard(r, world))[0]
        assert set(packed) == {"q", "k", "v", "o", "gate_up", "down"}
        assert all(isinstance(p, PackedWeight) for p in packed.values())

        def deq(w):
            if scheme == "int4-g128":
                return o.quantize_int4_group128(w).dequantized()
            if scheme == "fp8":
                return o.quantize_float(w, *o.E4M3, axis=0).dequantized()
            return o.quantize_integer(w, 8, True, 0).dequantized()

        # group-128 tables are held as f16 (a documented cast of the f32 tables);
        # the few fp8 codes below e4m3's normal range that keep more fraction
        # bits than an e4m3 subnormal are stored as the nearest e4m3 value
        tol = {"int4-g128": dict(rtol=1e-3, atol=1e-7), "fp8": dict(rtol=0, atol=1e-6),
               "int8": dict(rtol=0, atol=0)}[scheme]
        q_cols = o.split_heads(deq(blk.q_proj), r, world, cfg.num_heads, cfg.head_dim)
        np.testing.assert_allclose(packed["q"].dequantize().cpu().numpy(), q_cols, **tol)
        kv = o.split_heads(deq(blk.v_proj), r, world, cfg.num_kv_heads, cfg.head_dim)
        np.testing.assert_allclose(packed["v"].dequantize().cpu().numpy(), kv, **tol)
        want_o = o.split_input_dim(deq(blk.o_proj), r, world)
        np.testing.assert_allclose(packed["o"].dequantize().cpu().numpy(), want_o, **tol)
        want_d = o.split_input_dim(deq(blk.down_proj), r, world)
        np.testing.assert_allclose(packed["down"].dequantize().cpu().numpy(), want_d, **tol)
        gu = packed["gate_up"]
        assert gu.gate_up and gu.n == 2 * cfg.intermediate_size // world
        # gate/up pairs: the pair's columns are the oracle's gate and up shards
        # (rows interleaved), and its fused SiLU*up product with f32
        # activations is the f32 product of those columns
        gu_deq = gu.dequantize().cpu().numpy()
        np.testing.assert_allclose(gu_deq[:, 0::2],
                                   o.split_output_dim(deq(blk.gate_proj), r, world), **tol)
        np.testing.assert_allclose(gu_deq[:, 1::2],
                                   o.split_output_dim(deq(blk.up_proj), r, world), **tol)
        xt = torch.from_numpy(x).cuda()
        from ie_tpq.linear import qlinear

        got = qlinear(xt, gu).cpu().numpy()
        g, u = x @ gu_deq[:, 0::2], x @ gu_deq[:, 1::2]
        np.testing.assert_allclose(got, o.silu(g) * u, rtol=1e-3, atol=1e-4)
