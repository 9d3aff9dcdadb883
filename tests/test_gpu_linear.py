"""Quantized linear parity: ``qlinear`` (ie_qlinear through the C ABI) against
the oracle's dequantize-then-matmul (the reference's path,
ie/quant/weights.py:22-26 then ie/parallel/sharding.py:51-66).

Tolerances: f32 activations are compared tightly against an f64 product of
the weights the device actually holds (only accumulation order differs), and
against the reference's own f32 weights at the north-star bound
rtol 2e-2 / atol 2e-3; bf16 activations at that bound."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ie_tpq import formats as F
from ie_tpq import weights as W
from ie_tpq.linear import ALGO_GEMV, qlinear
from ie_tpq.packed import PackedWeight
from oracle import tpq_oracle as o

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3          # north-star tolerance for fp16/bf16 accumulate
TIGHT_RTOL, TIGHT_ATOL = 1e-4, 1e-5


def quantize(scheme, w):
    if scheme == "int8-k":
        return W.quantize_integer(w, F.INT8, 0), o.quantize_integer(w, 8, True, 0).dequantized()
    if scheme == "int8-n":
        return W.quantize_integer(w, F.INT8, 1), o.quantize_integer(w, 8, True, 1).dequantized()
    if scheme == "int8-t":
        return (W.quantize_integer(w, F.INT8, None),
                o.quantize_integer(w, 8, True, None).dequantized())
    if scheme == "int4-k":
        return W.quantize_integer(w, F.INT4, 0), o.quantize_integer(w, 4, True, 0).dequantized()
    if scheme == "int4-g128":
        return W.quantize_grouped(w), o.quantize_int4_group128(w).dequantized()
    if scheme == "fp8-k":
        return (W.quantize_float(w, F.FP8_E4M3, 0),
                o.quantize_float(w, *o.E4M3, axis=0).dequantized())
    if scheme == "fp8-n":
        return (W.quantize_float(w, F.FP8_E4M3, 1),
                o.quantize_float(w, *o.E4M3, axis=1).dequantized())
    raise KeyError(scheme)


SCHEMES = ["int8-k", "int8-n", "int8-t", "int4-k", "int4-g128", "fp8-k", "fp8-n"]


@pytest.mark.parametrize("scheme", SCHEMES)
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 17])
def test_f32_matches_the_dequantized_reference(scheme, m):
    k, n = 512, 96
    w = o.seeded_weight(k, n, seed=11)
    x = o.seeded_activations(m, k, seed=m)
    q, ref_w = quantize(scheme, w)
    p = q.packed()
    y = qlinear(torch.from_numpy(x).cuda(), p).cpu().numpy()
    dev_w = p.dequantize().cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(y, x.astype(np.float64) @ dev_w, rtol=TIGHT_RTOL, atol=TIGHT_ATOL)
    np.testing.assert_allclose(y, x @ ref_w, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("scheme", SCHEMES)
@pytest.mark.parametrize("m", [1, 4, 16])
def test_bf16_matches_within_the_north_star_tolerance(scheme, m):
    k, n = 1024, 256
    w = o.seeded_weight(k, n, seed=12)
    x = o.seeded_activations(m, k, seed=100 + m)
    q, ref_w = quantize(scheme, w)
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = qlinear(xb, q.packed()).float().cpu().numpy()
    want = xb.float().cpu().numpy() @ ref_w
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("scheme", ["int8-k", "int4-g128", "fp8-n", "int8-t"])
def test_gate_up_pairs_fuse_silu_times_up(scheme):
    k, n, m = 256, 64, 3
    g_w, u_w = o.seeded_weight(k, n, seed=21), o.seeded_weight(k, n, seed=22)
    x = o.seeded_activations(m, k, seed=23)
    gq, g_ref = quantize(scheme, g_w)
    uq, u_ref = quantize(scheme, u_w)
    pair = PackedWeight.pair_gate_up(gq.packed(), uq.packed())
    y = qlinear(torch.from_numpy(x).cuda(), pair).cpu().numpy()
    d = pair.dequantize("nk").cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(y, o.silu(x @ d[0::2].T) * (x @ d[1::2].T), rtol=1e-4, atol=1e-5)
    want = o.silu(x @ g_ref) * (x @ u_ref)
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)


def test_bias_and_residual_epilogue():
    k, n, m = 256, 48, 5
    w = o.seeded_weight(k, n, seed=31)
    x = o.seeded_activations(m, k, seed=32)
    res = o.seeded_activations(m, n, seed=33)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    q, ref_w = quantize("int8-k", w)
    y = qlinear(torch.from_numpy(x).cuda(), q.packed(), bias=torch.from_numpy(bias).cuda(),
                residual=torch.from_numpy(res).cuda()).cpu().numpy()
    np.testing.assert_allclose(y, res + (x @ ref_w + bias), rtol=1e-4, atol=1e-5)


def test_odd_row_counts_and_strided_inputs():
    k, n, m = 128, 6, 3
    w = o.seeded_weight(k, n, seed=41)
    x = o.seeded_activations(m, 2 * k, seed=42)
    q, ref_w = quantize("int8-n", w)
    xt = torch.from_numpy(x).cuda()[:, :k]      # row stride 2k
    y = qlinear(xt, q.packed(), algo=ALGO_GEMV).cpu().numpy()
    np.testing.assert_allclose(y, x[:, :k] @ ref_w, rtol=1e-4, atol=1e-5)


def test_zero_tokens_is_a_no_op():
    q, _ = quantize("int8-k", o.seeded_weight(64, 32, seed=43))
    y = qlinear(torch.empty((0, 64), device="cuda"), q.packed())
    assert y.shape == (0, 32)


def test_shape_mismatch_raises_value_error():
    q, _ = quantize("int8-k", o.seeded_weight(64, 32, seed=44))
    with pytest.raises(ValueError):
        qlinear(torch.zeros((2, 48), device="cuda"), q.packed())


def test_long_k_and_many_rows():
    """Llama-3-8B down_proj at TP=8 (K=1792, N=4096), decode batch 4, int4-g128."""
    k, n, m = 1792, 4096, 4
    w = o.seeded_weight(k, n, seed=51)
    x = o.seeded_activations(m, k, seed=52)
    q, ref_w = quantize("int4-g128", w)
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = qlinear(xb, q.packed()).float().cpu().numpy()
    np.testing.assert_allclose(y, xb.float().cpu().numpy() @ ref_w, rtol=RTOL, atol=ATOL)
