"""Attention pieces around the quantized projections: RoPE, KV-cache writes and
paged attention on the device.

These are not the quantized linear path; they sit between its projections
(q/k/v before, o after) exactly as in the reference's ``TorchBlock.forward``
(ie/model/torch_transformer.py:31-60), and are written with plain torch ops
(cuBLAS / SDPA underneath) or, for f16/bf16 models, the flash-attn kernels the
reference itself calls (ie/kernels/flash_backend.py:20-57).  The cache layout
is the reference's: ``[num_blocks * block_size, kv_heads, head_dim]`` with
``slot = block_table[pos // block_size] * block_size + pos % block_size``
(ie/kernels/torch_backend.py:6-10, ie/core/layout.py:57-64).
"""
from __future__ import annotations

import numpy as np

from .device import require_cuda

try:  # the reference's optional dependency (ie/kernels/flash_backend.py:5-13)
    from flash_attn import flash_attn_varlen_func, flash_attn_with_kvcache

    FLASH = True
except Exception:  # pragma: no cover - depends on the image
    flash_attn_varlen_func = flash_attn_with_kvcache = None
    FLASH = False

# flash-attn 2.8 rejects a paged KV cache whose page (block) size is not a
# multiple of 256 ("Paged KV cache block size must be divisible by 256").
PAGED_FLASH_BLOCK = 256


def allocate_kv_cache(num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                      device, dtype):
    """ie/kernels/torch_backend.py:6-10."""
    torch = require_cuda()
    shape = (num_blocks * block_size, num_kv_heads, head_dim)
    return (torch.zeros(shape, device=device, dtype=dtype),
            torch.zeros(shape, device=device, dtype=dtype))


def apply_rope(x, positions, cos, sin, halved: bool = False):
    """ie/layers/functional.py:34-61 (interleaved or halved), on device tensors."""
    torch = require_cuda()
    c = cos.index_select(0, positions).unsqueeze(1).to(x.dtype)
    s = sin.index_select(0, positions).unsqueeze(1).to(x.dtype)
    out = torch.empty_like(x)
    if halved:
        half = x.shape[-1] // 2
        left, right = x[..., :half], x[..., half:]
        out[..., :half] = left * c - right * s
        out[..., half:] = right * c + left * s
    else:
        even, odd = x[..., 0::2], x[..., 1::2]
        out[..., 0::2] = even * c - odd * s
        out[..., 1::2] = even * s + odd * c
    return out


def rope_write_kv(qkv, heads: int, kv_heads: int, head_dim: int, positions, cos, sin, slots,
                  k_cache, v_cache, halved: bool = False):
    """RoPE of q and k and the KV-cache write for the fused q|k|v projection's
    output ``qkv`` [tokens, (heads + 2 kv_heads) * head_dim] in one launch
    (``ie_rope_kv``); returns the rotated q [tokens, heads, head_dim].  Bitwise
    equal to ``apply_rope`` on q and k followed by ``write_kv``."""
    from . import _lib
    from .device import dtype_code

    torch = require_cuda()
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be a row-contiguous 2-D tensor")
    if k_cache.dtype != qkv.dtype or v_cache.dtype != qkv.dtype:
        raise ValueError("the caches must have the activations' dtype")
    for t, what in ((positions, "positions"), (slots, "slots")):
        if t.dtype != torch.long or not t.is_contiguous() or t.numel() != qkv.shape[0]:
            raise ValueError(f"{what} must be a contiguous int64 tensor of one entry per token")
    if not (cos.dtype == sin.dtype == torch.float32 and cos.is_contiguous()
            and sin.is_contiguous() and cos.shape[-1] * 2 == head_dim):
        raise ValueError("cos / sin must be contiguous f32 [max_position, head_dim / 2]")
    q = torch.empty((qkv.shape[0], heads, head_dim), dtype=qkv.dtype, device=qkv.device)
    _lib.check(_lib.lib().ie_rope_kv(
        qkv.data_ptr(), qkv.stride(0), dtype_code(qkv.dtype), qkv.shape[0], heads, kv_heads,
        head_dim, positions.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
        1 if halved else 0, slots.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.shape[0], q.data_ptr(), _lib.stream_ptr()), "rope_kv")
    return q


def write_kv(k, v, k_cache, v_cache, slots) -> None:
    """ie/kernels/reference.py:42-49 / torch_backend.py:13-16."""
    k_cache.index_copy_(0, slots, k.to(k_cache.dtype))
    v_cache.index_copy_(0, slots, v.to(v_cache.dtype))


def _gather(cache, table, context_len: int, block_size: int):
    torch = require_cuda()
    needed = (context_len + block_size - 1) // block_size
    if needed > table.shape[0]:
        raise IndexError(f"context of {context_len} needs {needed} blocks, "
                         f"table has {table.shape[0]}")
    offsets = torch.arange(block_size, device=cache.device)
    slots = (table[:needed, None] * block_size + offsets[None, :]).reshape(-1)
    return cache.index_select(0, slots[:context_len])


def paged_attention(q, k_cache, v_cache, block_tables, context_lens, query_lens,
                    block_size: int):
    """Causal attention of each sequence's queries over its cached context, f32
    softmax (ie/kernels/reference.py:65-80 and torch_backend.py:71-96).
    ``q`` [tokens, heads, hd]; ``block_tables`` a [seqs, width] device tensor."""
    torch = require_cuda()
    heads = q.shape[1]
    outs, start = [], 0
    for i, (ctx, ql) in enumerate(zip(context_lens, query_lens)):
        ctx, ql = int(ctx), int(ql)
        k = _gather(k_cache, block_tables[i], ctx, block_size)
        v = _gather(v_cache, block_tables[i], ctx, block_size)
        if heads != k.shape[1]:
            k = k.repeat_interleave(heads // k.shape[1], dim=1)
            v = v.repeat_interleave(heads // v.shape[1], dim=1)
        rows = torch.arange(ql, device=q.device)[:, None] + (ctx - ql)
        cols = torch.arange(ctx, device=q.device)[None, :]
        out = torch.nn.functional.scaled_dot_product_attention(
            q[start:start + ql].transpose(0, 1).unsqueeze(0).float(),
            k.transpose(0, 1).unsqueeze(0).float(), v.transpose(0, 1).unsqueeze(0).float(),
            attn_mask=(cols <= rows).unsqueeze(0))
        outs.append(out.squeeze(0).transpose(0, 1).to(q.dtype))
        start += ql
    return torch.cat(outs, dim=0)


def flash_decode(q, k_cache, v_cache, block_tables, context_lens, block_size: int,
                 scale: float):
    """One query token per sequence over paged caches (ie/kernels/flash_backend.py:20-33)."""
    view = lambda c: c.view(c.shape[0] // block_size, block_size, c.shape[1], c.shape[2])
    out = flash_attn_with_kvcache(q.unsqueeze(1), view(k_cache), view(v_cache),
                                  cache_seqlens=context_lens, block_table=block_tables,
                                  softmax_scale=scale, causal=True)
    return out.squeeze(1)


def flash_prefill(q, k, v, k_cache, v_cache, cu_q, cu_k, max_q: int, max_k: int,
                  paged_tables, block_size: int, scale: float):
    """Variable-length prefill (ie/kernels/flash_backend.py:36-57)."""
    if paged_tables is None:
        return flash_attn_varlen_func(q, k, v, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k,
                                      max_seqlen_q=max_q, max_seqlen_k=max_k,
                                      softmax_scale=scale, causal=True)
    view = lambda c: c.view(c.shape[0] // block_size, block_size, c.shape[1], c.shape[2])
    return flash_attn_varlen_func(q, view(k_cache), view(v_cache), cu_seqlens_q=cu_q,
                                  cu_seqlens_k=cu_k, max_seqlen_q=max_q, max_seqlen_k=max_k,
                                  softmax_scale=scale, causal=True, block_table=paged_tables)


def as_device_tables(block_tables, device):
    """A layout's block tables (lists padded with -1) as a long device tensor."""
    torch = require_cuda()
    arr = np.asarray(block_tables, dtype=np.int64)
    if arr.ndim == 1:
        arr = arr.reshape(1, -1)
    return torch.as_tensor(arr, device=device)
