"""Parity of the tcgen05 tensor-core path (algo=2) against the oracle.

The A operand is the weight dequantized to f16 in tensor memory (TMEM), so
each weight carries one extra rounding of at most half an ulp of f16 (2^-11
relative) before f32 accumulation; outputs are
held to the north-star tolerance rtol 2e-2 / atol 2e-3 against the
reference's f32 dequantize-then-matmul, and to the same bound against the
f32 weight-streaming kernel.  Split-K partials are summed in split order, so
repeated calls are bitwise identical."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq import formats as F
from ie_tpq import weights as W
from ie_tpq.comm import Communicator
from ie_tpq.linear import ALGO_GEMV, ALGO_TCGEN05, qlinear
from ie_tpq.packed import PackedWeight
from oracle import tpq_oracle as o
from tests.test_gpu_linear import quantize

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
SCHEMES = ["int4-g128", "int8-k", "int8-n", "fp8-n", "fp8-k", "int4-k", "int8-t"]


def status_bits() -> int:
    v = ctypes.c_uint32()
    _lib.check(_lib.lib().ie_kernel_status(ctypes.byref(v), 1))
    return v.value


@pytest.mark.parametrize("scheme", SCHEMES)
@pytest.mark.parametrize("m", [1, 2, 16, 17, 64, 130])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_matches_the_reference(scheme, m, dtype):
    k, n = 1024, 384
    w = o.seeded_weight(k, n, seed=200)
    x = o.seeded_activations(m, k, seed=201 + m)
    q, ref_w = quantize(scheme, w)
    p = q.packed()
    xt = torch.from_numpy(x).cuda().to(dtype)
    y = qlinear(xt, p, algo=ALGO_TCGEN05).float().cpu().numpy()
    want = xt.float().cpu().numpy() @ ref_w
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
    g = qlinear(xt, p, algo=ALGO_GEMV).float().cpu().numpy()
    np.testing.assert_allclose(y, g, rtol=RTOL, atol=ATOL)
    assert status_bits() == 0


@pytest.mark.parametrize("k,n,m", [(128, 96, 3), (4096, 4096, 16), (14336, 512, 16),
                                   (4096, 1024, 300), (2048, 6144, 64)])
def test_tc_shapes_and_split_k_are_deterministic(k, n, m):
    w = o.seeded_weight(k, n, seed=k + n)
    x = o.seeded_activations(m, k, seed=m)
    q = W.quantize_grouped(w)
    p = q.packed()
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y1 = qlinear(xt, p, algo=ALGO_TCGEN05)
    y2 = qlinear(xt, p, algo=ALGO_TCGEN05)
    assert torch.equal(y1, y2)
    want = xt.float().cpu().numpy() @ o.quantize_int4_group128(w).dequantized()
    np.testing.assert_allclose(y1.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    assert status_bits() == 0


@pytest.mark.parametrize("scheme", ["int4-g128", "int8-k", "fp8-n"])
def test_tc_gate_up_silu_bias_residual(scheme):
    k, n, m = 512, 256, 5
    g_w, u_w = o.seeded_weight(k, n, seed=31), o.seeded_weight(k, n, seed=32)
    x = o.seeded_activations(m, k, seed=33)
    gq, g_ref = quantize(scheme, g_w)
    uq, u_ref = quantize(scheme, u_w)
    pair = PackedWeight.pair_gate_up(gq.packed(), uq.packed())
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    xf = xt.float().cpu().numpy()
    res = torch.from_numpy(o.seeded_activations(m, n, seed=34)).cuda().to(torch.bfloat16)
    y = qlinear(xt, pair, residual=res, algo=ALGO_TCGEN05).float().cpu().numpy()
    want = res.float().cpu().numpy() + o.silu(xf @ g_ref) * (xf @ u_ref)
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
    q, ref_w = quantize(scheme, g_w)
    bias = torch.linspace(-1, 1, n, device="cuda")
    y = qlinear(xt, q.packed(), bias=bias, algo=ALGO_TCGEN05).float().cpu().numpy()
    np.testing.assert_allclose(y, xf @ ref_w + bias.cpu().numpy(), rtol=RTOL, atol=ATOL)


def test_tc_fused_allreduce_at_world_one_and_timeout():
    q = W.quantize_grouped(o.seeded_weight(4096, 1024, seed=40))
    p = q.packed()
    x = torch.from_numpy(o.seeded_activations(16, 4096, seed=41)).cuda().to(torch.bfloat16)
    res = torch.from_numpy(o.seeded_activations(16, 1024, seed=42)).cuda().to(torch.bfloat16)
    plain = qlinear(x, p, residual=res, algo=ALGO_TCGEN05)
    comm = Communicator(0, 1)
    try:
        for _ in range(3):
            fused = qlinear(x, p, residual=res, comm=comm, algo=ALGO_TCGEN05)
            assert torch.equal(plain, fused)
        comm.check()
    finally:
        comm.close()
    comm = Communicator.loopback(world_size=2, timeout_s=0.05)
    try:
        qlinear(x, p, residual=res, comm=comm, algo=ALGO_TCGEN05)
        with pytest.raises(_lib.TimeoutError_):
            comm.check()
        again = qlinear(x, p, residual=res, algo=ALGO_TCGEN05)
        assert torch.equal(plain, again)
    finally:
        comm.close()
    assert status_bits() == 0


def test_auto_routes_decode_batches_to_the_tensor_cores():
    q = W.quantize_grouped(o.seeded_weight(1024, 256, seed=50))
    p = q.packed()
    x = torch.from_numpy(o.seeded_activations(8, 1024, seed=51)).cuda().to(torch.bfloat16)
    assert torch.equal(qlinear(x, p), qlinear(x, p, algo=ALGO_TCGEN05))
    x1 = x[:1]
    assert torch.equal(qlinear(x1, p), qlinear(x1, p, algo=ALGO_TCGEN05))
    # f32 activations stay on the weight-streaming kernel
    xf = x1.float()
    assert torch.equal(qlinear(xf, p), qlinear(xf, p, algo=ALGO_GEMV))
