"""Tensor-parallel parity on one GPU: every rank's shard runs on the device,
partials are summed with the reference's rank-order ``all_reduce``, and the
result equals the reference's TP output (golden fixtures and the full-size
CPU case).  Also: the fused row-parallel + all-reduce entry point at world 1,
and the bounded peer wait ending in a timeout status (a loopback communicator
whose peer never pushes), after which the context stays usable."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq import formats as F
from ie_tpq import weights as W
from ie_tpq.comm import Communicator
from ie_tpq.linear import qlinear
from ie_tpq.sharding import ColumnParallelLinear, RowParallelLinear, Shard, all_reduce
from ie_tpq.tensor_parallel import ShardedMLP, rms_norm
from oracle import tpq_oracle as o

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


def test_list_all_reduce_is_the_reference_order_bitwise():
    parts = [o.seeded_activations(7, 33, seed=s) for s in range(4)]
    assert np.array_equal(all_reduce(parts), o.all_reduce(parts))


def test_rms_norm_matches_the_reference():
    x = o.seeded_activations(9, 896, seed=3)
    w = np.linspace(0.5, 1.5, 896).astype(np.float32)
    got = rms_norm(torch.from_numpy(x).cuda(), w).cpu().numpy()
    np.testing.assert_allclose(got, o.rms_norm(x, w), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("h", [4096, 8192, 1000, 13])
def test_rms_norm_vector_and_scalar_rows(h):
    """Hidden sizes that are multiples of 8 take the vector kernel (several
    chunks per thread at 8192); 1000 is one too (125 chunks); 13 takes the
    scalar loop.  bf16 in and out, compared with the f32 reference on the
    same rounded inputs; strided rows take the scalar loop as well."""
    x = o.seeded_activations(16, h, seed=h)
    w = np.linspace(0.5, 1.5, h).astype(np.float32)
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    want = o.rms_norm(xb.float().cpu().numpy(), w)
    got = rms_norm(xb, w).float().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=8e-3, atol=1e-5)   # one bf16 rounding
    wide = torch.zeros((16, h + 3), dtype=torch.bfloat16, device="cuda")
    wide[:, :h] = xb
    got = rms_norm(wide[:, :h], w).float().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=8e-3, atol=1e-5)
    xf = torch.from_numpy(x).cuda()
    np.testing.assert_allclose(rms_norm(xf, w).cpu().numpy(), o.rms_norm(x, w),
                               rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_sharded_mlp_matches_the_golden_tp_output(golden, world):
    x = golden["mlp_x"]
    # the fixture's weights are the reference's int8-dequantized f32 weights;
    # re-quantizing them with int8/axis 0 gives the same codes and scales
    # within an ulp, so the dequantized weights agree to f32 rounding
    qs = {name: W.quantize_integer(golden[f"mlp_{name}"], F.INT8)
          for name in ("gate", "up", "down")}
    for name in qs:
        np.testing.assert_allclose(qs[name].dequantized(), golden[f"mlp_{name}"], rtol=1e-6)
    xt = torch.from_numpy(x).cuda()
    partials = [ShardedMLP.from_weights(np.ones(64, np.float32), qs["gate"], qs["up"],
                                        qs["down"], Shard(r, world)).forward(xt)
                for r in range(world)]
    got = (xt + all_reduce(partials)).cpu().numpy()
    np.testing.assert_allclose(got, golden[f"mlp_out_{world}"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_full_size_cpu_case_tp2(golden_hashes, dtype):
    """hidden 896, intermediate 4864, 64 tokens, TP=2, int8 per-channel (axis 0)."""
    x, norm, gate, up, down = o.config1_inputs()
    qs = {n: W.quantize_integer(w, F.INT8) for n, w in (("gate", gate), ("up", up),
                                                        ("down", down))}
    xt = torch.from_numpy(x).cuda().to(dtype)
    parts = [ShardedMLP.from_weights(norm, qs["gate"], qs["up"], qs["down"],
                                     Shard(r, 2)).forward(xt) for r in range(2)]
    got = (xt.float() + all_reduce([p.float() for p in parts])).cpu().numpy()
    deq = {n: q.dequantized() for n, q in qs.items()}
    want = o.tp_mlp(xt.float().cpu().numpy(), norm, deq["gate"], deq["up"], deq["down"], 2)
    if dtype == torch.float32:
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
        assert float(np.sum(got.astype(np.float64))) == pytest.approx(
            golden_hashes["config1_out_tp2_sum"], rel=1e-4, abs=1e-2)
    else:
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL * 10)


@pytest.mark.parametrize("world", [2, 4])
def test_column_then_row_reproduces_the_unsharded_matmul(world):
    """tests/test_tensor_parallel.py:59-72 with quantized weights on the device."""
    x = o.seeded_activations(5, 256, seed=60)
    first = W.quantize_grouped(o.seeded_weight(256, 512, seed=61))
    second = W.quantize_grouped(o.seeded_weight(512, 256, seed=62))
    whole = (x @ first.dequantized()) @ second.dequantized()
    partials = []
    for r in range(world):
        sh = Shard(r, world)
        hidden = ColumnParallelLinear(first, sh).forward(x)
        partials.append(RowParallelLinear(second, sh).forward(hidden))
    np.testing.assert_allclose(all_reduce(partials), whole, rtol=2e-3, atol=2e-3)


def test_fused_allreduce_at_world_one_equals_the_plain_layer():
    comm = Communicator(0, 1)
    try:
        q = W.quantize_integer(o.seeded_weight(512, 256, seed=70), F.INT8)
        p = q.packed()
        x = torch.from_numpy(o.seeded_activations(6, 512, seed=71)).cuda()
        res = torch.from_numpy(o.seeded_activations(6, 256, seed=72)).cuda()
        plain = qlinear(x, p, residual=res)
        for _ in range(3):   # epochs advance; landing parity alternates
            fused = qlinear(x, p, residual=res, comm=comm)
            assert torch.equal(plain, fused)
        y = comm.all_reduce(res)
        assert torch.equal(y, res)
        comm.check()
    finally:
        comm.close()


@pytest.mark.parametrize("algo", ["oneshot", "twoshot"])
def test_fused_allreduce_protocols_at_world_one(algo):
    """At world 1 the two-shot owner path (every tile owned, nothing pushed to
    peers) must give the plain layer's result bit for bit, on both kernels."""
    from ie_tpq.comm import AR_ONESHOT, AR_TWOSHOT

    a = AR_TWOSHOT if algo == "twoshot" else AR_ONESHOT
    comm = Communicator(0, 1, algo=a)
    try:
        for dt, k, n, m in ((torch.float32, 512, 256, 6), (torch.bfloat16, 1024, 512, 40)):
            q = W.quantize_grouped(o.seeded_weight(k, n, seed=73))
            p = q.packed()
            x = torch.from_numpy(o.seeded_activations(m, k, seed=74)).cuda().to(dt)
            res = torch.from_numpy(o.seeded_activations(m, n, seed=75)).cuda().to(dt)
            bias = torch.from_numpy(o.seeded_activations(1, n, seed=76)[0]).cuda()
            plain = qlinear(x, p, residual=res, bias=bias)
            for _ in range(3):
                assert torch.equal(plain, qlinear(x, p, residual=res, bias=bias, comm=comm))
            big = torch.from_numpy(o.seeded_activations(64, 1000, seed=77)).cuda().to(dt)
            assert torch.equal(comm.all_reduce(big), big)
        comm.check()
    finally:
        comm.close()


def test_nvls_protocol_is_reported_unsupported():
    from ie_tpq.comm import AR_NVLS

    comm = Communicator(0, 1)
    try:
        with pytest.raises(RuntimeError, match="NVLS"):
            comm.all_reduce(torch.ones(4096, device="cuda"), algo=AR_NVLS)
    finally:
        comm.close()


@pytest.mark.parametrize("algo", ["oneshot", "twoshot"])
def test_peer_that_never_arrives_ends_in_a_timeout_status(algo):
    from ie_tpq.comm import AR_ONESHOT, AR_TWOSHOT

    comm = Communicator.loopback(world_size=2, timeout_s=0.05,
                                 algo=AR_TWOSHOT if algo == "twoshot" else AR_ONESHOT)
    try:
        q = W.quantize_integer(o.seeded_weight(256, 64, seed=80), F.INT8)
        p = q.packed()
        x = torch.from_numpy(o.seeded_activations(2, 256, seed=81)).cuda()
        qlinear(x, p, comm=comm)
        with pytest.raises(_lib.TimeoutError_):
            comm.check()
        comm.check()   # the status word was cleared
        # the context is still healthy: a normal layer runs and is correct
        y = qlinear(x, p).cpu().numpy()
        np.testing.assert_allclose(y, x.cpu().numpy() @ q.dequantized(), rtol=1e-4, atol=1e-5)
        comm.all_reduce(torch.ones(10000, device="cuda"))
        with pytest.raises(_lib.TimeoutError_):
            comm.check()
    finally:
        comm.close()


def test_communicator_rejects_oversized_requests():
    comm = Communicator(0, 1, max_bytes=1024)
    try:
        with pytest.raises(ValueError):
            comm.all_reduce(torch.ones(100000, device="cuda"))
    finally:
        comm.close()
