"""fp8 weights contracted natively with per-token fp8 activations
(``act_quant=IE_ACT_FP8_TOKEN``, BASELINE config 4's scheme) on the tensor
cores (tcgen05.mma kind::f8f6f4), against the oracle: the reference's
quantize_float(x, FP8_E4M3, axis=0) per token (``quantize_activations_fp8``)
and quantize_float(W, FP8_E4M3, axis=1) per output channel, both dequantized,
then an f32 matmul -- at the north-star rtol 2e-2 / atol 2e-3.  Shapes cover
single tiles, split-K (cluster and global partials), several token tiles,
per-tensor scales, a gate/up pair with SiLU, a residual, and the fused
all-reduce at world 1; the error cases follow the C ABI's rules."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq import formats as F
from ie_tpq import weights as W
from ie_tpq.linear import qlinear
from ie_tpq.packed import PackedWeight
from oracle import tpq_oracle as o

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
FP8 = _lib.IE_ACT_FP8_TOKEN


def oracle_act(x: np.ndarray) -> np.ndarray:
    return o.quantize_activations_fp8(x).dequantized()


@pytest.mark.parametrize("k,n,m", [(512, 384, 1), (1024, 256, 16), (8192, 1024, 16),
                                   (8192, 1024, 64), (4096, 512, 300), (14336, 512, 8),
                                   (2048, 4096, 1)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_native_fp8_matches_the_oracle(k, n, m, dtype):
    w = o.seeded_weight(k, n, seed=k + n)
    q = W.quantize_float(w, F.FP8_E4M3, 1)
    wd = o.quantize_float(w, *o.E4M3, axis=1).dequantized()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=m + 5)).cuda().to(dtype)
    y = qlinear(x, q.packed(), act_quant=FP8).float().cpu().numpy()
    want = oracle_act(x.float().cpu().numpy()) @ wd
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
    assert torch.equal(qlinear(x, q.packed(), act_quant=FP8), qlinear(x, q.packed(),
                                                                       act_quant=FP8))


def test_per_tensor_scale_residual_and_pairs():
    k, n, m = 2048, 512, 24
    w = o.seeded_weight(k, n, seed=3)
    q = W.quantize_float(w, F.FP8_E4M3, None)
    wd = o.quantize_float(w, *o.E4M3, axis=None).dequantized()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=4)).cuda().to(torch.bfloat16)
    res = torch.from_numpy(o.seeded_activations(m, n, seed=6)).cuda().to(torch.bfloat16)
    xa = oracle_act(x.float().cpu().numpy())
    y = qlinear(x, q.packed(), residual=res, act_quant=FP8).float().cpu().numpy()
    np.testing.assert_allclose(y, res.float().cpu().numpy() + xa @ wd, rtol=RTOL, atol=ATOL)
    # gate/up pair: silu(x@g) * (x@u) on the same e4m3 activations
    g = W.quantize_float(o.seeded_weight(k, n, seed=7), F.FP8_E4M3, 1)
    u = W.quantize_float(o.seeded_weight(k, n, seed=8), F.FP8_E4M3, 1)
    pair = PackedWeight.pair_gate_up(g.packed(), u.packed())
    gd = o.quantize_float(o.seeded_weight(k, n, seed=7), *o.E4M3, axis=1).dequantized()
    ud = o.quantize_float(o.seeded_weight(k, n, seed=8), *o.E4M3, axis=1).dequantized()
    got = qlinear(x, pair, act_quant=FP8).float().cpu().numpy()
    from tests.test_gpu_llama_shapes import check_silu_mul

    check_silu_mul(got, xa @ gd, xa @ ud)


def test_fused_allreduce_world_one():
    from ie_tpq.comm import Communicator

    k, n, m = 4096, 768, 16
    w = o.seeded_weight(k, n, seed=9)
    q = W.quantize_float(w, F.FP8_E4M3, 1)
    wd = o.quantize_float(w, *o.E4M3, axis=1).dequantized()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=10)).cuda().to(torch.bfloat16)
    comm = Communicator(0, 1, max_bytes=1 << 22)
    try:
        y = qlinear(x, q.packed(), comm=comm, act_quant=FP8).float().cpu().numpy()
        comm.check()
    finally:
        comm.close()
    np.testing.assert_allclose(y, oracle_act(x.float().cpu().numpy()) @ wd, rtol=RTOL, atol=ATOL)


def test_zero_rows_and_errors():
    k, n = 512, 256
    q = W.quantize_float(o.seeded_weight(k, n, seed=1), F.FP8_E4M3, 1)
    x = torch.zeros((3, k), dtype=torch.bfloat16, device="cuda")
    x[1] = torch.linspace(-3, 3, k, device="cuda")
    y = qlinear(x, q.packed(), act_quant=FP8).float().cpu().numpy()
    assert np.all(y[0] == 0) and np.all(y[2] == 0) and np.any(y[1] != 0)
    # per-K fp8 scales, integer weights and f32 activations are refused
    with pytest.raises(ValueError):
        qlinear(x, W.quantize_float(o.seeded_weight(k, n, seed=1), F.FP8_E4M3, 0).packed(),
                act_quant=FP8)
    with pytest.raises(ValueError):
        qlinear(x, W.quantize_integer(o.seeded_weight(k, n, seed=1), F.INT8, 1).packed(),
                act_quant=FP8)
    with pytest.raises(ValueError):
        qlinear(x.float(), q.packed(), act_quant=FP8)
