"""The activation pre-pass of the tensor-core kernel against the in-loop
conversion it replaces.

With a workspace, a launch whose activations need converting (bf16, or the
RMS norm folded in) first has its CTAs write the MMA's f16 operand once into
the workspace (each CTA a slice, then a grid barrier); without one, every CTA
converts each x tile it loads.  Both apply the same arithmetic in the same
order -- bf16 -> f16 saturating, or f16((x * rinv) * w) with the same per-token
rinv -- so on shapes whose plan has a single K split the two outputs are
bitwise equal.  Both are also held to the oracle (rms_norm, then the
reference's f32 dequantize-then-matmul) at rtol 2e-2 / atol 2e-3."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq.linear import ALGO_TCGEN05, build_args, qlinear
from ie_tpq.packed import PackedWeight
from oracle import tpq_oracle as o
from tests.test_gpu_linear import quantize
from tests.test_gpu_llama_shapes import check_silu_mul

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


def in_loop(x, p, out, **kw):
    """The same call with no workspace: no pre-pass and no split-K."""
    a = build_args(x, p, out, algo=ALGO_TCGEN05, **kw)
    a.workspace = None
    a.workspace_bytes = 0
    _lib.check(_lib.lib().ie_qlinear(ctypes.byref(a), _lib.stream_ptr()), "qlinear")
    return out


def workspace_bytes(x, p, out, **kw) -> int:
    a = build_args(x, p, out, algo=ALGO_TCGEN05, **kw)
    return _lib.lib().ie_qlinear_workspace_size(ctypes.byref(a))


def check_pre_pass(scheme, k, n, m, dtype, norm):
    q, ref_w = quantize(scheme, o.seeded_weight(k, n, seed=k + m))
    p = q.packed()
    xf = o.seeded_activations(m, k, seed=m + 3)
    if norm:   # rows of different magnitudes: the norm rescales each one
        xf = xf * np.linspace(0.5, 6.0, m, dtype=np.float32)[:, None]
    x = torch.from_numpy(xf.astype(np.float32)).cuda().to(dtype)
    nw = torch.linspace(0.5, 1.5, k, device="cuda") if norm else None
    kw = dict(norm_weight=nw) if norm else {}
    pre = qlinear(x, p, algo=ALGO_TCGEN05, **kw)
    # the plan converts the activations once: the workspace holds them
    assert workspace_bytes(x, p, pre, **kw) >= m * k * 2
    loop = in_loop(x, p, torch.empty_like(pre), **kw)
    assert torch.equal(pre, loop)
    xin = x.float().cpu().numpy()
    if norm:
        xin = o.rms_norm(xin, nw.cpu().numpy())
    np.testing.assert_allclose(pre.float().cpu().numpy(), xin @ ref_w, rtol=RTOL, atol=ATOL)


# Folded RMS norm above 16 tokens takes the pre-pass.  K = 1024 (int4, four
# 128-K sub-stages per TMA stage) and K = 512 (8-bit, two) give two TMA stages
# along K, too few for the plan to split K, so both calls run one split.
@pytest.mark.parametrize("scheme,k", [("int4-g128", 1024), ("int8-k", 512), ("fp8-n", 512),
                                      ("int4-k", 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m", [17, 40, 130])
def test_pre_pass_with_norm_equals_in_loop_conversion(scheme, k, dtype, m):
    check_pre_pass(scheme, k, 1536, m, dtype, True)


# Plain bf16 activations take the pre-pass when the conversion the CTAs would
# repeat is large: 128 row tiles of 130 tokens over K = 4096 (one split: 128
# units fill one wave).
@pytest.mark.parametrize("scheme,k", [("int4-g128", 4096), ("int8-k", 4096), ("fp8-n", 4096)])
def test_pre_pass_bf16_equals_in_loop_conversion(scheme, k):
    check_pre_pass(scheme, k, 16384, 130, torch.bfloat16, False)


@pytest.mark.parametrize("m", [1, 16, 64, 200])
def test_pre_pass_with_split_k_and_gate_up(m):
    """Shapes whose plan splits K (cluster or global partials) and a gate/up
    pair with SiLU: the pre-pass path against the oracle, and repeatable."""
    k, n = 8192, 1024
    g, gw = quantize("int4-g128", o.seeded_weight(k, n, seed=1))
    u, uw = quantize("int4-g128", o.seeded_weight(k, n, seed=2))
    pair = PackedWeight.pair_gate_up(g.packed(), u.packed())
    x = torch.from_numpy(o.seeded_activations(m, k, seed=4)).cuda().to(torch.bfloat16)
    nw = torch.linspace(0.5, 1.5, k, device="cuda")
    y1 = qlinear(x, pair, norm_weight=nw)
    y2 = qlinear(x, pair, norm_weight=nw)
    assert torch.equal(y1, y2)
    xin = o.rms_norm(x.float().cpu().numpy(), nw.cpu().numpy())
    check_silu_mul(y1.float().cpu().numpy(), xin @ gw, xin @ uw)
    d, dw = quantize("int4-g128", o.seeded_weight(n, 4096, seed=5))
    h = y1.contiguous()
    res = torch.from_numpy(o.seeded_activations(m, 4096, seed=6)).cuda().to(torch.bfloat16)
    y = qlinear(h, d.packed(), residual=res).float().cpu().numpy()
    want = res.float().cpu().numpy() + h.float().cpu().numpy() @ dw
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
