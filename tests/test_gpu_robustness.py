"""Edge cases of the tensor-core kernel's state and number ranges.

* A caller workspace whose ticket region holds leftovers (as a launch that gave
  up on an expired wait would leave it) must not change the next result: every
  ticket word carries the tag of the launch that counted it, and a word with
  another tag counts as zero.
* bf16 activations beyond f16's range reach the tensor cores saturated to
  +-65504 (the activation operand is f16): outputs stay finite.
* Small-magnitude weights (std 1e-3 and 1e-4, group scales near f16's
  subnormal range) still meet rtol 2e-2 / atol 2e-3 against the oracle.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq.linear import ALGO_TCGEN05, build_args, qlinear
from oracle import tpq_oracle as o
from tests.test_gpu_linear import quantize

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


@pytest.mark.parametrize("scheme,k,n,m", [("int4-g128", 4096, 1024, 64),
                                          ("int8-k", 4096, 6144, 16)])
def test_stale_tickets_in_a_caller_workspace_are_ignored(scheme, k, n, m):
    w = o.seeded_weight(k, n, seed=3)
    q, ref_w = quantize(scheme, w)
    p = q.packed()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=4)).cuda().to(torch.bfloat16)
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    need = _lib.lib().ie_qlinear_workspace_size(
        ctypes.byref(build_args(x, p, out, algo=ALGO_TCGEN05)))
    if need == 0:
        pytest.skip("this shape reduces its splits inside a cluster (no tickets)")
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    # the ticket words follow the 256 bytes of barrier and generation words;
    # every ticket counted already: counted as such, the first split to arrive
    # would finalize its tile from partial sums
    tickets = ws[256:256 + 4 * 64].view(torch.int32)
    tickets.fill_(1)
    y = qlinear(x, p, workspace=ws, algo=ALGO_TCGEN05).float().cpu().numpy()
    want = x.float().cpu().numpy() @ ref_w
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
    tickets.fill_(7)
    y2 = qlinear(x, p, workspace=ws, algo=ALGO_TCGEN05).float().cpu().numpy()
    assert np.array_equal(y, y2)
    # leftovers tagged by an earlier launch on this workspace (its tag is one
    # below the current generation's): ignored too
    gen = int(ws[8:12].view(torch.int32).item())
    tickets.fill_(((gen - 1) % 0xFFFFFF + 1) << 8 | 1)
    y3 = qlinear(x, p, workspace=ws, algo=ALGO_TCGEN05).float().cpu().numpy()
    assert np.array_equal(y, y3)


def test_bf16_activations_beyond_f16_range_saturate():
    k, n, m = 1024, 256, 4
    q, ref_w = quantize("int8-n", o.seeded_weight(k, n, seed=5))
    x = o.seeded_activations(m, k, seed=6)
    x[0, 7] = 1.0e5     # representable in bf16, not in f16
    x[2, 100] = -3.0e5
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = qlinear(xb, q.packed(), algo=ALGO_TCGEN05, out_dtype=torch.float32).cpu().numpy()
    assert np.all(np.isfinite(y))
    # rows without an out-of-range value are unaffected
    want = xb.float().cpu().numpy() @ ref_w
    np.testing.assert_allclose(y[[1, 3]], want[[1, 3]], rtol=RTOL, atol=ATOL)
    # the clamped rows equal the product with the saturated activations, up to
    # the f16 rounding of the dequantized weight (2^-12 relative) that the
    # 65504-sized term carries
    xs = np.clip(xb.float().cpu().numpy(), -65504.0, 65504.0)
    big = 65504.0 * float(np.abs(ref_w).max()) * 2.0 ** -10
    np.testing.assert_allclose(y[[0, 2]], (xs @ ref_w)[[0, 2]], rtol=RTOL, atol=big)


@pytest.mark.parametrize("std", [1e-3, 1e-4])
@pytest.mark.parametrize("scheme", ["int4-g128", "int8-k", "fp8-n"])
def test_small_magnitude_weights(std, scheme):
    k, n, m = 2048, 512, 16
    w = o.seeded_weight(k, n, seed=9, std=std)
    q, ref_w = quantize(scheme, w)
    xb = torch.from_numpy(o.seeded_activations(m, k, seed=10)).cuda().to(torch.bfloat16)
    y = qlinear(xb, q.packed(), algo=ALGO_TCGEN05).float().cpu().numpy()
    want = xb.float().cpu().numpy() @ ref_w
    np.testing.assert_allclose(y, want, rtol=RTOL, atol=ATOL)
