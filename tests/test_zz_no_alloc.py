"""ie_qlinear_noalloc, called through the C ABI: the tensor-core quantized
linear with its split-K partials, tile tickets and pre-converted activations
in the library's static device array instead of a caller workspace -- for callers that cannot
allocate device memory when they run a layer.  Two calls in a row must each
match ie_qlinear (caller workspace, the same kernel and split plan) and the
CPU oracle's dequantize-then-matmul within the north-star tolerance
rtol 2e-2 / atol 2e-3, equal each other bitwise, and leave the device's free
memory unchanged.

The file name sorts last so that the module also runs after every other GPU
test in one process; it passes alone in a fresh process as well."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ie_tpq import _lib
from ie_tpq import weights as W
from ie_tpq.linear import ALGO_TCGEN05, build_args, qlinear
from ie_tpq.packed import PackedWeight
from oracle import tpq_oracle as o
from tests.test_gpu_linear import quantize

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


def noalloc(a) -> int:
    return _lib.lib().ie_qlinear_noalloc(ctypes.byref(a), _lib.stream_ptr())


def status_bits() -> int:
    v = ctypes.c_uint32()
    _lib.check(_lib.lib().ie_kernel_status(ctypes.byref(v), 1))
    return v.value


def split_k_bytes(a) -> int:
    return _lib.lib().ie_qlinear_workspace_size(ctypes.byref(a))


# Token counts above 32: smaller batches reduce their K splits inside a
# thread-block cluster and need no scratch, so these shapes are the ones that
# exercise the static array.
@pytest.mark.parametrize("scheme,k,n,m", [
    ("int4-g128", 4096, 1024, 64),
    ("int4-g128", 14336, 512, 48),
    ("int8-k", 4096, 1024, 64),
    ("fp8-n", 2048, 768, 40),
    ("int4-k", 2048, 512, 64),
])
def test_two_calls_in_a_row_match_the_workspace_entry_point(scheme, k, n, m):
    w = o.seeded_weight(k, n, seed=k + n + m)
    q, ref_w = quantize(scheme, w)
    p = q.packed()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=m + 7)).cuda().to(torch.bfloat16)
    res = torch.from_numpy(o.seeded_activations(m, n, seed=m + 8)).cuda().to(torch.bfloat16)
    want = qlinear(x, p, residual=res, algo=ALGO_TCGEN05).float()
    oracle = res.float().cpu().numpy() + x.float().cpu().numpy() @ ref_w
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
            for _ in range(2)]
    args = [build_args(x, p, out, residual=res, algo=ALGO_TCGEN05) for out in outs]
    # the first call on a device looks the array up (the module is resident by
    # then: qlinear above ran a kernel of the same library); measure after it
    _lib.check(noalloc(args[0]), "qlinear_noalloc")
    torch.cuda.synchronize()
    outs[0].fill_(float("nan"))
    free_before = torch.cuda.mem_get_info()[0]
    for a in args:
        assert 0 < split_k_bytes(a) <= _lib.IE_QLINEAR_NOALLOC_SCRATCH_BYTES
        _lib.check(noalloc(a), "qlinear_noalloc")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    for out in outs:
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, want.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(got, oracle, rtol=RTOL, atol=ATOL)
    assert torch.equal(outs[0], outs[1])
    assert status_bits() == 0


def test_gate_up_pair_with_silu():
    k, n, m = 4096, 1024, 64
    pair = PackedWeight.pair_gate_up(quantize("int4-g128", o.seeded_weight(k, n, seed=1))[0].packed(),
                                     quantize("int4-g128", o.seeded_weight(k, n, seed=2))[0].packed())
    x = torch.from_numpy(o.seeded_activations(m, k, seed=3)).cuda().to(torch.bfloat16)
    want = qlinear(x, pair, algo=ALGO_TCGEN05).float().cpu().numpy()
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        a = build_args(x, pair, out, silu_mul=True, algo=ALGO_TCGEN05)
        _lib.check(noalloc(a), "qlinear_noalloc")
        np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    assert status_bits() == 0


def test_fused_rms_norm():
    k, n, m = 4096, 1024, 64
    p = W.quantize_grouped(o.seeded_weight(k, n, seed=11)).packed()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=12) * 4).cuda().to(torch.bfloat16)
    nw = torch.linspace(0.5, 1.5, k, device="cuda")
    want = qlinear(x, p, norm_weight=nw, algo=ALGO_TCGEN05)
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        a = build_args(x, p, out, norm_weight=nw, algo=ALGO_TCGEN05)
        assert split_k_bytes(a) > 0
        _lib.check(noalloc(a), "qlinear_noalloc")
        assert torch.equal(out, want)
    assert status_bits() == 0


def test_plans_beyond_the_static_scratch_run_a_plan_that_fits():
    """A shape whose preferred plan needs more scratch than the array holds runs
    the best plan that fits (without split-K, or also without the activation
    pre-pass) instead of failing.  Against ie_qlinear with a workspace (the
    split plan: only the f32 summation order and so at most a last-place bf16
    rounding differ) and against the oracle on sampled columns."""
    k, n, m = 8192, 4096, 256
    w = o.seeded_weight(k, n, seed=9)
    p = W.quantize_grouped(w).packed()
    x = torch.from_numpy(o.seeded_activations(m, k, seed=10)).cuda().to(torch.bfloat16)
    want = qlinear(x, p, algo=ALGO_TCGEN05).float().cpu().numpy()
    cols = np.sort(np.random.default_rng(11).choice(n, size=256, replace=False))
    oracle = x.float().cpu().numpy() @ o.quantize_int4_group128(w[:, cols]).dequantized()
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    a = build_args(x, p, out, algo=ALGO_TCGEN05)
    assert split_k_bytes(a) > _lib.IE_QLINEAR_NOALLOC_SCRATCH_BYTES
    for _ in range(2):
        _lib.check(noalloc(a), "qlinear_noalloc")
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-3)
        np.testing.assert_allclose(got[:, cols], oracle, rtol=RTOL, atol=ATOL)
    assert status_bits() == 0


def test_paths_other_than_the_tensor_cores_are_unsupported():
    q, _ = quantize("int8-k", o.seeded_weight(256, 128, seed=5))
    p = q.packed()
    x = torch.zeros((4, 256), dtype=torch.float32, device="cuda")
    out = torch.empty((4, 128), dtype=torch.float32, device="cuda")
    assert noalloc(build_args(x, p, out)) == _lib.IE_ERR_UNSUPPORTED
    empty = torch.empty((0, 256), dtype=torch.bfloat16, device="cuda")
    assert noalloc(build_args(empty, p, out[:0].to(torch.bfloat16))) == _lib.IE_OK
