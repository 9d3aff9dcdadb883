"""The fused RoPE + KV-cache write (``ie_rope_kv``) against the unfused steps
it replaces: ``apply_rope`` on q and k and ``write_kv`` (the reference's
ie/layers/functional.py:34-61 and ie/kernels/torch_backend.py:13-16 as device
tensor arithmetic) -- bitwise for bf16, f16 and f32, interleaved and halved
rotations, a strided q|k|v row and scattered slots -- and against the oracle's
f32 RoPE within the activation type's rounding."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ie_tpq.attention import apply_rope, rope_write_kv, write_kv
from oracle import model_oracle as mo

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("halved", [False, True])
@pytest.mark.parametrize("tokens,heads,kv,hd", [(16, 32, 8, 128), (5, 14, 2, 64), (1, 4, 4, 16)])
def test_fused_equals_unfused(dtype, halved, tokens, heads, kv, hd):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(tokens * 7 + heads)
    width = (heads + 2 * kv) * hd
    big = torch.randn((tokens, width + 64), generator=gen, device="cuda").to(dtype)
    qkv = big[:, 32:32 + width]                    # a strided row, as a column slice
    max_pos = 4096
    cos_np, sin_np = mo.rope_tables(max_pos, hd, 500000.0)
    cos = torch.from_numpy(cos_np).cuda()
    sin = torch.from_numpy(sin_np).cuda()
    positions = torch.randint(0, max_pos, (tokens,), generator=gen, device="cuda")
    slots = torch.randperm(4 * tokens, generator=gen, device="cuda")[:tokens]
    kc = torch.zeros((4 * tokens, kv, hd), dtype=dtype, device="cuda")
    vc = torch.zeros_like(kc)
    q = rope_write_kv(qkv, heads, kv, hd, positions, cos, sin, slots, kc, vc, halved)
    qn, kn = heads * hd, kv * hd
    q_ref = apply_rope(qkv[:, :qn].reshape(tokens, heads, hd), positions, cos, sin, halved)
    k_ref = apply_rope(qkv[:, qn:qn + kn].reshape(tokens, kv, hd), positions, cos, sin, halved)
    kc_ref, vc_ref = torch.zeros_like(kc), torch.zeros_like(vc)
    write_kv(k_ref, qkv[:, qn + kn:].reshape(tokens, kv, hd), kc_ref, vc_ref, slots)
    assert torch.equal(q, q_ref)
    assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)
    # the oracle's f32 rotation (ie/layers/functional.py:34-61)
    pos = positions.cpu().numpy()
    want = mo.apply_rope(qkv[:, :qn].float().cpu().numpy().reshape(tokens, heads, hd), pos,
                         cos_np, sin_np, halved)
    tol = {torch.float32: 1e-6, torch.float16: 2e-3, torch.bfloat16: 2e-2}[dtype]
    np.testing.assert_allclose(q.float().cpu().numpy(), want, rtol=tol, atol=tol)


def test_slots_outside_the_cache_write_nothing():
    tokens, heads, kv, hd = 3, 2, 1, 8
    qkv = torch.randn((tokens, (heads + 2 * kv) * hd), device="cuda")
    cos_np, sin_np = mo.rope_tables(16, hd)
    cos, sin = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()
    kc = torch.zeros((4, kv, hd), device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, -1, 99], device="cuda")
    positions = torch.tensor([1, 2, 3], device="cuda")
    rope_write_kv(qkv, heads, kv, hd, positions, cos, sin, slots, kc, vc)
    assert torch.count_nonzero(kc[1:]) == 0 and torch.count_nonzero(vc[1:]) == 0
    assert torch.count_nonzero(vc[0]) > 0


def test_shape_errors():
    qkv = torch.zeros((2, 10), device="cuda")
    cos = torch.zeros((4, 4), device="cuda")
    pos = torch.zeros(2, dtype=torch.long, device="cuda")
    kc = torch.zeros((4, 1, 8), device="cuda")
    with pytest.raises(ValueError):
        rope_write_kv(qkv, 2, 1, 8, pos, cos, cos, pos, kc, kc)   # width 10 < 32
