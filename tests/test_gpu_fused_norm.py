"""Parity of the RMS norm folded into the tensor-core GEMM (IE_EPI_RMS_NORM)
against the oracle: ``rms_norm`` (ie/layers/functional.py:6-8) followed by the
reference's f32 dequantize-then-matmul.

The fused call scales each x tile by the token's 1/sqrt(mean(x^2) + eps) and
the norm weight while converting it for the tensor cores, so the normalised
activation is rounded once, to f16; the two-kernel path rounds it to the
activation type first.  The fused call is held to the north-star tolerance
rtol 2e-2 / atol 2e-3 against the oracle, and to twice that against the
two-kernel path (which carries the extra bf16 rounding), and repeated
fused calls are bitwise identical (the per-token sums of squares and the
split-K reduction run in a fixed order)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq import weights as W
from ie_tpq.comm import Communicator
from ie_tpq.linear import ALGO_GEMV, ALGO_TCGEN05, build_args, fused_norm_ok, qlinear
from ie_tpq.packed import PackedWeight
from ie_tpq.tensor_parallel import rms_norm
from oracle import tpq_oracle as o
from tests.test_gpu_linear import quantize

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


def status_bits() -> int:
    v = ctypes.c_uint32()
    _lib.check(_lib.lib().ie_kernel_status(ctypes.byref(v), 1))
    return v.value


def norm_weight(k: int, seed: int) -> np.ndarray:
    return (0.5 + np.random.default_rng(seed).random(k)).astype(np.float32)


def activations(m: int, k: int, seed: int) -> np.ndarray:
    # residual-stream-like rows: a spread of per-token magnitudes, so the
    # normalisation changes every row by a different factor
    x = o.seeded_activations(m, k, seed=seed)
    return (x * np.linspace(0.25, 8.0, m, dtype=np.float32)[:, None]).astype(np.float32)


@pytest.mark.parametrize("scheme", ["int4-g128", "int8-k", "int8-n", "fp8-n", "int4-k"])
@pytest.mark.parametrize("m", [1, 5, 16, 64, 130])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_norm_matches_the_reference(scheme, m, dtype):
    k, n, eps = 1024, 384, 1e-6
    q, ref_w = quantize(scheme, o.seeded_weight(k, n, seed=300))
    p = q.packed()
    nw = norm_weight(k, 301)
    xt = torch.from_numpy(activations(m, k, 302 + m)).cuda().to(dtype)
    nwt = torch.from_numpy(nw).cuda()
    assert fused_norm_ok(xt, p)
    y = qlinear(xt, p, norm_weight=nwt, norm_eps=eps, algo=ALGO_TCGEN05).float().cpu().numpy()
    want = o.rms_norm(xt.float().cpu().numpy(), nw, eps) @ ref_w
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
    # the two-kernel path carries the extra rounding of the normalised x to the
    # activation type, so the two calls are held to twice the bound
    two = qlinear(rms_norm(xt, nwt, eps), p, algo=ALGO_TCGEN05).float().cpu().numpy()
    np.testing.assert_allclose(y, two, rtol=2 * RTOL, atol=2 * ATOL)
    assert status_bits() == 0


# Llama-3 shapes: qkv (global split-K), o-like (cluster split-K), multiple
# token tiles, a 8192-wide hidden size
@pytest.mark.parametrize("k,n,m", [(4096, 6144, 16), (4096, 4096, 16), (4096, 1024, 300),
                                   (8192, 1024, 8), (4096, 2048, 48)])
def test_fused_norm_shapes_and_splits_are_deterministic(k, n, m):
    eps = 1e-5
    w = o.seeded_weight(k, n, seed=k + n)
    p = W.quantize_grouped(w).packed()
    nw = norm_weight(k, m)
    nwt = torch.from_numpy(nw).cuda()
    xt = torch.from_numpy(activations(m, k, seed=m + 1)).cuda().to(torch.bfloat16)
    y1 = qlinear(xt, p, norm_weight=nwt, norm_eps=eps, algo=ALGO_TCGEN05)
    y2 = qlinear(xt, p, norm_weight=nwt, norm_eps=eps, algo=ALGO_TCGEN05)
    assert torch.equal(y1, y2)
    want = o.rms_norm(xt.float().cpu().numpy(), nw, eps) @ o.quantize_int4_group128(w).dequantized()
    np.testing.assert_allclose(y1.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    assert status_bits() == 0


@pytest.mark.parametrize("scheme", ["int4-g128", "int8-k", "fp8-n"])
def test_fused_norm_gate_up_silu_residual(scheme):
    k, n, m, eps = 512, 256, 5, 1e-6
    gq, g_ref = quantize(scheme, o.seeded_weight(k, n, seed=41))
    uq, u_ref = quantize(scheme, o.seeded_weight(k, n, seed=42))
    pair = PackedWeight.pair_gate_up(gq.packed(), uq.packed())
    nw = norm_weight(k, 43)
    xt = torch.from_numpy(activations(m, k, seed=44)).cuda().to(torch.bfloat16)
    res = torch.from_numpy(o.seeded_activations(m, n, seed=45)).cuda().to(torch.bfloat16)
    y = qlinear(xt, pair, residual=res, norm_weight=torch.from_numpy(nw).cuda(), norm_eps=eps,
                algo=ALGO_TCGEN05).float().cpu().numpy()
    h = o.rms_norm(xt.float().cpu().numpy(), nw, eps)
    want = res.float().cpu().numpy() + o.silu(h @ g_ref) * (h @ u_ref)
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
    assert status_bits() == 0


def test_fused_norm_with_the_fused_allreduce_at_world_one():
    k, n, m = 4096, 1024, 16
    p = W.quantize_grouped(o.seeded_weight(k, n, seed=50)).packed()
    nwt = torch.from_numpy(norm_weight(k, 51)).cuda()
    xt = torch.from_numpy(activations(m, k, seed=52)).cuda().to(torch.bfloat16)
    res = torch.from_numpy(o.seeded_activations(m, n, seed=53)).cuda().to(torch.bfloat16)
    plain = qlinear(xt, p, residual=res, norm_weight=nwt, algo=ALGO_TCGEN05)
    comm = Communicator(0, 1)
    try:
        for _ in range(2):
            fused = qlinear(xt, p, residual=res, norm_weight=nwt, comm=comm, algo=ALGO_TCGEN05)
            assert torch.equal(plain, fused)
        comm.check()
    finally:
        comm.close()
    assert status_bits() == 0


@pytest.mark.parametrize("scheme", ["int4-g128", "int8-k", "fp8-n", "int4-k"])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_weight_streaming_decode_folds_the_norm(scheme, m, dtype):
    """The decode GEMV (at most two tokens) stages x for the whole K once per
    CTA and applies the RMS norm there in f32: rms_norm then the reference's
    f32 matmul.  f32 activations are held to the bound of the other f32
    weight-streaming tests (2e-3: int4-g128 group tables are f16 on the
    device), bf16 ones to the north-star tolerance."""
    k, n, eps = 2048, 384, 1e-6
    q, ref_w = quantize(scheme, o.seeded_weight(k, n, seed=310))
    p = q.packed()
    nw = norm_weight(k, 311)
    xt = torch.from_numpy(activations(m, k, 312 + m)).cuda().to(dtype)
    res = torch.from_numpy(o.seeded_activations(m, n, seed=313)).cuda().to(dtype)
    y = qlinear(xt, p, residual=res, norm_weight=torch.from_numpy(nw).cuda(), norm_eps=eps,
                algo=ALGO_GEMV, out_dtype=torch.float32 if dtype == torch.float32 else None)
    h = o.rms_norm(xt.float().cpu().numpy(), nw, eps)
    want = res.float().cpu().numpy() + h @ ref_w
    rtol, atol = (2e-3, 2e-3) if dtype == torch.float32 else (RTOL, ATOL)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=rtol, atol=atol)


def test_weight_streaming_decode_gate_up_pairs():
    k, n, m, eps = 1024, 256, 1, 1e-6
    gq, g_ref = quantize("int4-g128", o.seeded_weight(k, n, seed=320))
    uq, u_ref = quantize("int4-g128", o.seeded_weight(k, n, seed=321))
    pair = PackedWeight.pair_gate_up(gq.packed(), uq.packed())
    nw = norm_weight(k, 322)
    xt = torch.from_numpy(activations(m, k, seed=323)).cuda()
    y = qlinear(xt, pair, norm_weight=torch.from_numpy(nw).cuda(), norm_eps=eps,
                algo=ALGO_GEMV).cpu().numpy()
    h = o.rms_norm(xt.cpu().numpy(), nw, eps)
    np.testing.assert_allclose(y, o.silu(h @ g_ref) * (h @ u_ref), rtol=2e-3, atol=2e-3)


def test_fused_norm_rejections():
    k, n, m = 1024, 256, 4
    p = W.quantize_grouped(o.seeded_weight(k, n, seed=60)).packed()
    nwt = torch.from_numpy(norm_weight(k, 61)).cuda()
    xt = torch.from_numpy(activations(m, k, seed=62)).cuda().to(torch.bfloat16)
    # the weight-streaming kernel folds the norm only for at most two tokens
    with pytest.raises(ValueError):
        qlinear(xt, p, norm_weight=nwt, algo=ALGO_GEMV)
    # f32 activations cannot take the tensor-core path
    assert not fused_norm_ok(xt.float(), p)
    with pytest.raises(RuntimeError):
        qlinear(xt.float(), p, norm_weight=nwt)
    with pytest.raises(ValueError):
        qlinear(xt, p, norm_weight=nwt[:-1])
    # flag without a weight, through the C ABI
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    a = build_args(xt, p, out, algo=ALGO_TCGEN05)
    a.epilogue |= _lib.IE_EPI_RMS_NORM
    assert _lib.lib().ie_qlinear(ctypes.byref(a), _lib.stream_ptr()) == _lib.IE_ERR_INVALID


@pytest.mark.parametrize("scheme", ["int4-g128", "int8"])
def test_linear_stack_folds_both_norms(scheme):
    from ie_tpq.sharding import Shard
    from ie_tpq.stack import DecoderShape, LinearStack, synthetic_layer

    shape = DecoderShape(hidden=1024, heads=8, kv_heads=2, head_dim=128, intermediate=2048,
                         layers=2)
    layers = [synthetic_layer(shape, scheme, Shard(0, 1), seed=70 + i) for i in range(2)]
    x = torch.from_numpy(activations(16, shape.hidden, seed=72)).cuda().to(torch.bfloat16)
    fused = LinearStack(shape, layers, batch=16)
    plain = LinearStack(shape, layers, batch=16, fuse_norm=False)
    fused.norm.copy_(torch.from_numpy(norm_weight(shape.hidden, 73)))
    plain.norm.copy_(fused.norm)
    y_f = fused.forward(x)
    y_p = plain.forward(x)
    # qkv (or q, k, v) and gate/up take the norm; no rms_norm launches remain
    per_layer = 4 if scheme == "int4-g128" else 6
    assert fused.launches_per_step == per_layer * 2
    assert plain.launches_per_step == (per_layer + 2) * 2
    # Each layer adds into the bf16 residual stream, whose rounding step is set
    # by the row's magnitude (the rows here span 0.25x to 8x), so beside twice
    # the per-call bound one bf16 ulp of the row's largest value may flip.
    yf, yp = y_f.float().cpu().numpy(), y_p.float().cpu().numpy()
    ulp = np.abs(yp).max(axis=1, keepdims=True) * 2.0 ** -7
    assert np.all(np.abs(yf - yp) <= 2 * RTOL * np.abs(yp) + 2 * ATOL + ulp)
    fused.x_in.copy_(x)
    fused.capture()
    fused.replay()
    torch.cuda.synchronize()
    assert torch.equal(fused.x_out, y_f)
    assert status_bits() == 0
