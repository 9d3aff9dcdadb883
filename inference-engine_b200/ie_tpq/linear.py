"""The quantized linear call: one packed shard times a token batch on the GPU,
with the epilogue fused in and, for a row-parallel layer, the all-reduce fused
in as well (``comm=``).  This is the device form of the reference's
``x @ W_shard`` (ie/parallel/sharding.py:51-66) and of the projections in
``TorchBlock.forward`` (ie/model/torch_transformer.py:36-38,60) and
``torch_backend.swiglu`` (ie/kernels/torch_backend.py:125-127).
"""
from __future__ import annotations

import ctypes

from . import _lib
from .device import dtype_code, require_cuda
from .packed import PackedWeight

ALGO_AUTO, ALGO_GEMV, ALGO_TCGEN05 = 0, 1, 2

# One workspace per device, grown on demand: split-K partials and tile
# tickets, and the converted activations of the pre-pass.  Zero-filled once;
# its barrier and generation words stay consistent by themselves and the
# tickets carry each launch's tag, so consecutive calls on one stream share it;
# calls on concurrent streams must pass their own ``workspace=``.
_WORKSPACE: dict = {}


def shared_workspace(nbytes: int, device):
    torch = require_cuda()
    key = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WORKSPACE.get(key)
    if ws is None or ws.numel() < nbytes:
        size = max(nbytes, 2 * ws.numel() if ws is not None else 1 << 20)
        ws = torch.zeros(size, dtype=torch.uint8, device=device)
        _WORKSPACE[key] = ws
    return ws


# Largest token batch for which folding the RMS norm into the next GEMM beats
# a separate rms_norm launch.  Each CTA of the fused call first reads its token
# rows from L2 for the sums of squares and then scales every x tile it
# converts; on B200 with Llama-3-8B shapes (qkv + gate/up, int4-g128) the
# two fused calls cost 3.6 / 4.6 us more than the plain GEMMs at 8 / 16 tokens
# against 6.8 / 7.2 us for two rms_norm launches, and 10.6 us more at 24-32.
FUSED_NORM_MAX_TOKENS = 16


def fused_norm_ok(x, w: PackedWeight) -> bool:
    """Whether ``qlinear(x, w, norm_weight=...)`` can fold the RMS norm in:
    the tensor-core path (bf16/f16 rows, 16-byte aligned, K a multiple of 128)
    with the activations contracted as given (not quantized per token)."""
    torch = require_cuda()
    return (x.dim() == 2 and x.dtype in (torch.bfloat16, torch.float16) and w.k % 128 == 0
            and not w.act_quant
            and x.stride(1) == 1 and x.data_ptr() % 16 == 0 and (x.stride(0) * 2) % 16 == 0)


def fuse_norm_pays(x, w: PackedWeight) -> bool:
    """``fused_norm_ok`` and a batch small enough for the fold to be faster."""
    return x.shape[0] <= FUSED_NORM_MAX_TOKENS and fused_norm_ok(x, w)


def build_args(x, w: PackedWeight, out, *, bias=None, residual=None, silu_mul=False,
               algo=ALGO_AUTO, workspace=None, norm_weight=None,
               norm_eps: float = 1e-6, act_quant: int = 0) -> _lib.QLinearArgs:
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [tokens, K], got shape {tuple(x.shape)}")
    if x.shape[1] != w.k:
        raise ValueError(f"x has K={x.shape[1]} but the weight has K={w.k}")
    if x.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("x and out must be contiguous along their last dimension")
    epi = 0
    if bias is not None:
        epi |= _lib.IE_EPI_BIAS
    if residual is not None:
        epi |= _lib.IE_EPI_RESIDUAL
        if residual.dtype != out.dtype or residual.stride(1) != 1:
            raise ValueError("residual must match out's dtype and be row-contiguous")
    if silu_mul:
        epi |= _lib.IE_EPI_SILU_MUL
    if norm_weight is not None:
        epi |= _lib.IE_EPI_RMS_NORM
        if norm_weight.dtype != require_cuda().float32 or norm_weight.numel() != w.k or \
                not norm_weight.is_contiguous():
            raise ValueError(f"norm_weight must be a contiguous f32 [{w.k}] tensor")
    a = _lib.QLinearArgs()
    a.w = w.qweight()
    a.m = x.shape[0]
    a.act_dtype = dtype_code(x.dtype)
    a.out_dtype = dtype_code(out.dtype)
    a.x = x.data_ptr()
    a.ldx = x.stride(0)
    a.out = out.data_ptr()
    a.ldo = out.stride(0)
    a.bias = bias.data_ptr() if bias is not None else None
    a.residual = residual.data_ptr() if residual is not None else None
    a.ldr = residual.stride(0) if residual is not None else 0
    a.epilogue = epi
    a.norm_weight = norm_weight.data_ptr() if norm_weight is not None else None
    a.norm_eps = float(norm_eps)
    a.act_quant = int(act_quant)
    a.algo = algo
    a.workspace = workspace.data_ptr() if workspace is not None else None
    a.workspace_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    return a


def qlinear(x, w: PackedWeight, *, bias=None, residual=None, silu_mul: bool | None = None,
            out=None, out_dtype=None, comm=None, algo: int = ALGO_AUTO, stream=None,
            workspace=None, norm_weight=None, norm_eps: float = 1e-6,
            act_quant: int | None = None, reduce_algo: int | None = None):
    """``y = x @ deq(W)`` on the GPU; ``comm`` fuses the row-parallel all-reduce
    (protocol ``reduce_algo``, default ``comm.algo``).

    x: CUDA tensor ``[M, K]`` (bf16 / f16 / f32).  bias: f32 ``[N]``.  residual:
    ``[M, N]`` of the output dtype, added after the reduction.  A gate/up pair
    weight returns ``silu(gate) * up`` of shape ``[M, N/2]``.  ``norm_weight``
    (f32 ``[K]``) folds ``rms_norm(x, norm_weight, norm_eps)`` in front of the
    product (ie/layers/functional.py:6-8); it needs the tensor-core path
    (``fused_norm_ok``), or the weight-streaming path (``algo=ALGO_GEMV`` or
    f32 x) for at most two tokens, and raises otherwise.  ``act_quant=IE_ACT_FP8_TOKEN``
    (fp8 weights with per-N or per-tensor scales) quantizes each token of x to
    e4m3 with its own scale and contracts the e4m3 codes on the tensor cores.
    """
    torch = require_cuda()
    if silu_mul is None:
        silu_mul = w.gate_up
    if act_quant is None:   # the weight's scheme decides ("fp8-native": per-token e4m3)
        act_quant = w.act_quant
    out_dtype = out_dtype or x.dtype
    cols = w.out_features if silu_mul else w.n
    if out is None:
        out = torch.empty((x.shape[0], cols), dtype=out_dtype, device=x.device)
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        bias = bias.to(torch.float32).contiguous()
    if norm_weight is not None and (norm_weight.dtype != torch.float32
                                    or not norm_weight.is_contiguous()):
        norm_weight = norm_weight.to(torch.float32).contiguous()
    a = build_args(x, w, out, bias=bias, residual=residual, silu_mul=silu_mul, algo=algo,
                   norm_weight=norm_weight, norm_eps=norm_eps, act_quant=act_quant)
    need = _lib.lib().ie_qlinear_workspace_size(ctypes.byref(a))
    if need:
        ws = workspace if workspace is not None else shared_workspace(need, x.device)
        if ws.numel() * ws.element_size() < need:
            raise ValueError(f"workspace of {ws.numel() * ws.element_size()} bytes < {need} needed")
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel() * ws.element_size()
    s = _lib.stream_ptr(stream)
    if comm is None:
        _lib.check(_lib.lib().ie_qlinear(ctypes.byref(a), s), "qlinear")
    else:
        algo = comm.algo if reduce_algo is None else int(reduce_algo)
        _lib.check(_lib.lib().ie_qlinear_allreduce(comm.handle, ctypes.byref(a), algo, s),
                   "qlinear_allreduce")
    return out
