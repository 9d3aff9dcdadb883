"""Tensor-parallel blocks on the GPU -- the device form of the reference's
ie/parallel/tensor_parallel.py for the linear path.

``ShardedMLP`` holds one rank's gate/up column shards (packed as gate/up row
pairs so the SiLU*up product is fused into the GEMM epilogue) and its down
row shard.  ``forward(x)`` returns the rank's partial like the reference
(ie/parallel/tensor_parallel.py:54-56); ``forward(x, comm=c)`` returns
``x + all_reduce(partials)`` (tensor_parallel.py:73) with the residual add and
the all-reduce fused into the down projection's epilogue.

``kv_heads_per_rank`` keeps the reference's check (tensor_parallel.py:76-79).
"""
from __future__ import annotations

import numpy as np

from . import _lib
from .device import dtype_code, require_cuda
from .packed import PackedWeight
from .sharding import Shard, split_input_dim, split_output_dim
from .weights import QuantizedWeight


def kv_heads_per_rank(config, world_size: int) -> int:
    """ie/parallel/tensor_parallel.py:76-79."""
    if config.num_kv_heads % world_size:
        raise ValueError(f"{config.num_kv_heads} kv heads do not divide across {world_size} ranks")
    return config.num_kv_heads // world_size


def rms_norm(x, weight, eps: float = 1e-6, out_dtype=None):
    """ie/layers/functional.py:6-8 on the GPU (``ie_rms_norm``)."""
    torch = require_cuda()
    if x.dim() != 2:
        raise ValueError("rms_norm takes [tokens, hidden]")
    w = weight if isinstance(weight, torch.Tensor) else torch.from_numpy(
        np.ascontiguousarray(weight, dtype=np.float32))
    w = w.to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    _lib.check(_lib.lib().ie_rms_norm(x.data_ptr(), x.stride(0), dtype_code(x.dtype), w.data_ptr(),
                                      out.data_ptr(), out.stride(0), dtype_code(out.dtype),
                                      x.shape[0], x.shape[1], float(eps), _lib.stream_ptr()),
               "rms_norm")
    return out


def _pack(w, device=None) -> PackedWeight:
    if isinstance(w, PackedWeight):
        return w
    if isinstance(w, QuantizedWeight):
        return PackedWeight.from_quantized(w, device=device)
    raise TypeError("expected a QuantizedWeight or PackedWeight")


class ShardedMLP:
    """One rank's share of the SwiGLU MLP (ie/parallel/tensor_parallel.py:46-56)."""

    def __init__(self, norm, gate, up, down, shard: Shard, eps: float = 1e-6,
                 device=None) -> None:
        torch = require_cuda()
        self.shard = shard
        self.eps = eps
        self.norm = torch.as_tensor(np.asarray(norm, dtype=np.float32)).cuda() \
            if not isinstance(norm, torch.Tensor) else norm.cuda().float()
        g = _pack(split_output_dim(gate, shard), device)
        u = _pack(split_output_dim(up, shard), device)
        self.gate_up = PackedWeight.pair_gate_up(g, u)
        self.down = _pack(split_input_dim(down, shard), device)

    def forward(self, x, comm=None):
        """Partial ``(silu(n@g) * (n@u)) @ d`` (comm=None), or ``x + sum of partials``."""
        from .linear import fuse_norm_pays, qlinear

        if fuse_norm_pays(x, self.gate_up):
            hidden = qlinear(x, self.gate_up, silu_mul=True, norm_weight=self.norm,
                             norm_eps=self.eps)
        else:
            hidden = qlinear(rms_norm(x, self.norm, self.eps), self.gate_up, silu_mul=True)
        if comm is None:
            return qlinear(hidden, self.down, out_dtype=x.dtype)
        return qlinear(hidden, self.down, residual=x, comm=comm, out_dtype=x.dtype)
