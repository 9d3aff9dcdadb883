"""Parity of the tensor-core kernel at the Llama-3-8B projection shapes the
benchmark runs: TP=1 and a TP=8 shard, decode batches 1, 16, 64 and 256,
int4 group-128 weights N(0, 0.02), bf16 activations.

Two checks per case:
  * against the CPU oracle (the reference's group-128 quantizer and f32
    dequantize-then-matmul) on 384 seeded output columns -- group tables are
    per output column, so the oracle quantizes exactly those columns of the
    f32 weight -- at the north-star rtol 2e-2 / atol 2e-3;
  * every output column against an f32 product with the device's own
    dequantized weight (``ie_dequantize``, bit-exact against the oracle in
    tests/test_gpu_pack.py), same tolerance.
Projections: qkv (RMS norm folded in), o (+ residual), gate/up (pair, fused
SiLU*up, norm folded in) and down (+ residual).  For gate/up the tolerance
applies to the two GEMM outputs and is carried through SiLU*up
(``check_silu_mul``)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ie_tpq.linear import qlinear
from ie_tpq.packed import PackedWeight, quantize_on_device
from oracle import tpq_oracle as o

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
COLS = 384
H, I, Q, KV = 4096, 14336, 4096, 1024


def shapes(tp: int):
    """(name, K, N) of one rank's projections; gate/up N counts both halves."""
    return (("qkv", H, (Q + 2 * KV) // tp), ("o", Q // tp, H), ("gate_up", H, 2 * I // tp),
            ("down", I // tp, H))


_cache: dict = {}


def weights(name: str, k: int, n: int):
    """(f32 weight on the device, packed weight) for a projection shape; gate/up
    is two weights of n/2 columns packed as row pairs."""
    key = (name, k, n)
    if key not in _cache:
        _cache.clear()
        torch.cuda.empty_cache()
        gen = torch.Generator(device="cuda")
        gen.manual_seed(k * 7 + n)
        if name == "gate_up":
            g = torch.randn((k, n // 2), generator=gen, device="cuda") * 0.02
            u = torch.randn((k, n // 2), generator=gen, device="cuda") * 0.02
            packed = PackedWeight.pair_gate_up(quantize_on_device(g, "int4-g128"),
                                               quantize_on_device(u, "int4-g128"))
            _cache[key] = ((g, u), packed)
        else:
            w = torch.randn((k, n), generator=gen, device="cuda") * 0.02
            _cache[key] = (w, quantize_on_device(w, "int4-g128"))
    return _cache[key]


def oracle_cols(w_dev, cols):
    sub = w_dev[:, torch.as_tensor(cols, device=w_dev.device)].cpu().numpy()
    return o.quantize_int4_group128(sub).dequantized()


def check(got, want):
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), (int(bad.sum()), float(err.max()))


def check_silu_mul(got, g, u):
    """SiLU(g) * u from the kernel against the same of the f32 products g, u.

    The tolerance applies to the GEMM outputs g and u (each within
    ATOL + RTOL * |.|) and is carried through SiLU * up to first order: where
    u is near zero and SiLU(g) is a few units, an error on u inside its own
    tolerance moves the product by up to |SiLU(g)| times that."""
    sg = o.silu(g)
    sig = 1.0 / (1.0 + np.exp(-g))       # d/dg silu(g) = sigmoid(g) * (1 + g * (1 - sigmoid(g)))
    dsg = sig * (1.0 + g * (1.0 - sig))
    want = sg * u
    tol = (np.abs(dsg * u) * (ATOL + RTOL * np.abs(g)) + np.abs(sg) * (ATOL + RTOL * np.abs(u)))
    err = np.abs(got - want)
    bad = err > tol + ATOL + RTOL * np.abs(want)
    assert not bad.any(), (int(bad.sum()), float(err.max()))


@pytest.mark.parametrize("tp", [1, 8])
@pytest.mark.parametrize("m", [1, 16, 64, 256])
@pytest.mark.parametrize("proj", ["qkv", "o", "gate_up", "down"])
def test_llama_shard_shape(tp, m, proj):
    name, k, n = next(s for s in shapes(tp) if s[0] == proj)
    w, packed = weights(name, k, n)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(m + 31 * tp)
    x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
    xf = x.float().cpu().numpy()
    rng = np.random.default_rng(m + tp)
    norm = name in ("qkv", "gate_up") and m <= 16
    nw = torch.linspace(0.5, 1.5, k, device="cuda") if norm else None
    xin = o.rms_norm(xf, nw.cpu().numpy()) if norm else xf
    if name == "gate_up":
        y = qlinear(x, packed, norm_weight=nw).float().cpu().numpy()
        half = n // 2
        cols = np.sort(rng.choice(half, size=min(COLS, half), replace=False))
        check_silu_mul(y[:, cols], xin @ oracle_cols(w[0], cols), xin @ oracle_cols(w[1], cols))
        deq = packed.dequantize().cpu().numpy()          # [K, 2 * half], rows interleaved
        check_silu_mul(y, xin @ deq[:, 0::2], xin @ deq[:, 1::2])
        return
    res = None
    if name in ("o", "down"):
        res = torch.randn((m, n), generator=gen, device="cuda").to(torch.bfloat16)
    y = qlinear(x, packed, residual=res, norm_weight=nw).float().cpu().numpy()
    rf = res.float().cpu().numpy() if res is not None else 0.0
    cols = np.sort(rng.choice(n, size=min(COLS, n), replace=False))
    want = xin @ oracle_cols(w, cols)
    if res is not None:
        want = rf[:, cols] + want
    check(y[:, cols], want)
    full = xin @ packed.dequantize().cpu().numpy()
    check(y, rf + full if res is not None else full)
