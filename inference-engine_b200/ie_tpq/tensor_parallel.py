"""Tensor-parallel transformer block on the GPU -- the API of the reference's
ie/parallel/tensor_parallel.py with quantized, packed shards.

The constructors keep the reference's signatures: ``ShardedAttention(block,
shard)``, ``ShardedMLP(block, shard)`` and ``TensorParallelBlock(block,
world_size)`` take a reference-style ``TransformerBlock`` (attributes
``attn_norm``, ``q_proj`` ... ``down_proj`` as ``[K, N]`` arrays, optional
``q_bias`` / ``k_bias`` / ``v_bias`` / ``q_norm`` / ``k_norm``, and a
``config`` with the head counts and ``norm_eps``).  Dense weights are
quantized on the device with ``scheme`` (default int8 with the reference's
per-output-channel axis) before they are sharded, as ``quantize_transformer``
followed by ``split_*`` would do; ``QuantizedWeight`` / ``PackedWeight``
attributes are sharded as they are.

``forward`` returns the rank's partial like the reference
(tensor_parallel.py:26-43,54-56); ``TensorParallelBlock.forward`` sums the
partials in rank order (``all_reduce``) and adds the residual
(tensor_parallel.py:65-73).  With one process per GPU, ``forward(..., comm=c)``
instead returns ``x + all_reduce(partials)`` with the residual and the
all-reduce fused into the o / down projection's epilogue.

NumPy inputs run in f32 (the weight-streaming kernel) and come back as NumPy;
NumPy KV caches are updated in place at the written slots, as the reference's
``write_kv`` does.  Torch CUDA inputs keep their dtype (bf16 / f16 take the
tensor-core kernel).  Deviations from the reference's TP attention, which
drops them: q/k/v biases are sharded with their columns and applied, and an
optional per-head q/k RMS norm is applied (ie/model/torch_transformer.py:36-44);
both are absent (zero / None) in a random-init block, so results agree.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np

from . import _lib
from .attention import apply_rope, paged_attention, write_kv
from .device import dtype_code, require_cuda
from .packed import PackedWeight, concat_rows
from .sharding import Shard, all_reduce, split_heads, split_input_dim, split_output_dim
from .weights import QuantizedWeight

PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def kv_heads_per_rank(config, world_size: int) -> int:
    """ie/parallel/tensor_parallel.py:76-79."""
    if config.num_kv_heads % world_size:
        raise ValueError(f"{config.num_kv_heads} kv heads do not divide across {world_size} ranks")
    return config.num_kv_heads // world_size


def rms_norm(x, weight, eps: float = 1e-6, out_dtype=None):
    """ie/layers/functional.py:6-8 on the GPU (``ie_rms_norm``), f32 arithmetic."""
    torch = require_cuda()
    if x.dim() != 2:
        raise ValueError("rms_norm takes [tokens, hidden]")
    w = weight if isinstance(weight, torch.Tensor) else torch.from_numpy(
        np.ascontiguousarray(weight, dtype=np.float32))
    w = w.to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    if x.shape[0] == 0:
        return out
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


def _own(p: PackedWeight) -> PackedWeight:
    """A column shard that does not keep the whole weight alive: a row slice
    of packed codes is a view of the full array, so it is copied out."""
    base = p.codes._base
    if base is None or base.numel() == p.codes.numel():
        return p
    return PackedWeight(fmt=p.fmt, axis=p.axis, k=p.k, n=p.n, codes=p.codes.clone(),
                        scale=p.scale.clone(), zero=p.zero.clone() if p.zero is not None else None,
                        int4_symmetric=p.int4_symmetric, gate_up=p.gate_up,
                        unrepresentable=p.unrepresentable, act_quant=p.act_quant)


def _f32(v, device):
    """A host vector (or None) as a contiguous f32 device tensor."""
    if v is None:
        return None
    torch = require_cuda()
    t = v if isinstance(v, torch.Tensor) else torch.from_numpy(np.asarray(v, dtype=np.float32))
    return t.to(device=device, dtype=torch.float32).contiguous()


MLP_PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def quantized_block(block, scheme: str = "int8", axis: int | None = 0,
                    names: tuple = PROJECTIONS):
    """A view of ``block`` whose projections ``names`` (all seven by default)
    are quantized (reference tables, computed on the device) and whose other
    attributes are shared.  Projections that are already quantized or packed
    are kept."""
    from .quant_model import quantize_for_device

    attrs = {}
    for name in names:
        w = getattr(block, name)
        attrs[name] = w if isinstance(w, (QuantizedWeight, PackedWeight)) else \
            quantize_for_device(np.asarray(w, dtype=np.float32), scheme, axis)
    for name in ("config", "attn_norm", "mlp_norm", "q_bias", "k_bias", "v_bias", "q_norm",
                 "k_norm"):
        attrs[name] = getattr(block, name, None)
    return SimpleNamespace(**attrs)


def _is_quantized(block) -> bool:
    return all(isinstance(getattr(block, n), (QuantizedWeight, PackedWeight)) for n in PROJECTIONS)


def _to_device(x, device):
    """(CUDA tensor, came-from-numpy)."""
    torch = require_cuda()
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device), True
    return (x if x.is_cuda else x.to(device)), False


class ShardedAttention:
    """One rank's attention heads (ie/parallel/tensor_parallel.py:12-43): q/k/v
    head-sharded column shards, the o projection a row shard."""

    def __init__(self, block, shard: Shard, *, scheme: str = "int8", axis: int | None = 0,
                 device=None) -> None:
        torch = require_cuda()
        if not _is_quantized(block):
            block = quantized_block(block, scheme, axis)
        config = block.config
        self.config = config
        self.shard = shard
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        hd = config.head_dim
        self.num_heads = config.num_heads // shard.world_size
        self.num_kv_heads = config.num_kv_heads // shard.world_size
        self.norm = _f32(block.attn_norm, self.device)
        self.eps = float(config.norm_eps)
        q = _own(_pack(split_heads(block.q_proj, shard, config.num_heads, hd), self.device))
        k = _own(_pack(split_heads(block.k_proj, shard, config.num_kv_heads, hd), self.device))
        v = _own(_pack(split_heads(block.v_proj, shard, config.num_kv_heads, hd), self.device))
        self.q_proj, self.k_proj, self.v_proj = q, k, v
        # one GEMM for q|k|v when their tables live on N (per-N, group-128)
        self.qkv = concat_rows([q, k, v]) if q.axis in (_lib.IE_AXIS_N, _lib.IE_AXIS_GROUP128) \
            else None
        self.o_proj = _pack(split_input_dim(block.o_proj, shard), self.device)
        cols = lambda heads: shard.slice_of(heads)

        def bias(b, heads):
            if b is None:
                return None
            sl = cols(heads)
            return _f32(np.asarray(b, dtype=np.float32)[sl.start * hd:sl.stop * hd], self.device)

        self.q_bias = bias(getattr(block, "q_bias", None), config.num_heads)
        self.k_bias = bias(getattr(block, "k_bias", None), config.num_kv_heads)
        self.v_bias = bias(getattr(block, "v_bias", None), config.num_kv_heads)
        # the fused projection's bias, q|k|v in row order (None without biases)
        self.qkv_bias = (torch.cat([self.q_bias, self.k_bias, self.v_bias]).contiguous()
                         if self.q_bias is not None else None)
        self.q_norm = _f32(getattr(block, "q_norm", None), self.device)
        self.k_norm = _f32(getattr(block, "k_norm", None), self.device)
        self.rope_halved = bool(getattr(config, "rope_halved", False))

    def _norm_in(self, x, first):
        from .linear import fuse_norm_pays

        if fuse_norm_pays(x, first):
            return x, self.norm
        return rms_norm(x, self.norm, self.eps), None

    def fused_qkv(self, x):
        """The q|k|v projection as one GEMM output ``[T, (heads + 2 kv_heads) * hd]``
        when the rank's q, k and v share one packed weight and no per-head
        q / k norm follows (the input of ``rope_write_kv``); else None."""
        from .linear import qlinear

        if self.qkv is None or self.q_norm is not None:
            return None
        h, nw = self._norm_in(x, self.qkv)
        return qlinear(h, self.qkv, bias=self.qkv_bias, norm_weight=nw, norm_eps=self.eps)

    def project_qkv(self, x):
        """q, k, v ``[T, heads, hd]`` of this rank for hidden states x (device)."""
        from .linear import qlinear

        hd = self.config.head_dim
        h, nw = self._norm_in(x, self.qkv if self.qkv is not None else self.q_proj)
        qn, kn = self.num_heads * hd, self.num_kv_heads * hd
        if self.qkv is not None:
            y = qlinear(h, self.qkv, bias=self.qkv_bias, norm_weight=nw, norm_eps=self.eps)
            q, k, v = y[:, :qn], y[:, qn:qn + kn], y[:, qn + kn:]
        else:
            q = qlinear(h, self.q_proj, bias=self.q_bias, norm_weight=nw, norm_eps=self.eps)
            k = qlinear(h, self.k_proj, bias=self.k_bias, norm_weight=nw, norm_eps=self.eps)
            v = qlinear(h, self.v_proj, bias=self.v_bias, norm_weight=nw, norm_eps=self.eps)
        q = q.reshape(-1, self.num_heads, hd)
        k = k.reshape(-1, self.num_kv_heads, hd)
        v = v.reshape(-1, self.num_kv_heads, hd)
        if self.q_norm is not None:
            q = rms_norm(q.reshape(-1, hd), self.q_norm, self.eps).reshape(q.shape)
            k = rms_norm(k.reshape(-1, hd), self.k_norm, self.eps).reshape(k.shape)
        return q, k, v

    def forward(self, x, layout, k_cache, v_cache, cos, sin, block_size: int, *, comm=None):
        """The rank's partial ``attention(x) @ o_shard`` (``comm=None``), or
        ``x + all_reduce(partials)`` with the reduction fused (``comm``)."""
        from .linear import qlinear

        torch = require_cuda()
        xt, was_numpy = _to_device(x, self.device)
        q, k, v = self.project_qkv(xt)
        positions = torch.as_tensor(np.asarray(layout.positions), device=self.device,
                                    dtype=torch.long)
        cos_t = _f32(cos, self.device)
        sin_t = _f32(sin, self.device)
        q = apply_rope(q, positions, cos_t, sin_t, self.rope_halved)
        k = apply_rope(k, positions, cos_t, sin_t, self.rope_halved)
        slots_np = np.asarray(layout.slot_mapping, dtype=np.int64)
        if len(slots_np) != k.shape[0]:
            raise ValueError(f"{len(slots_np)} slots for {k.shape[0]} tokens")
        slots = torch.as_tensor(slots_np, device=self.device)
        numpy_cache = isinstance(k_cache, np.ndarray)
        kc = torch.from_numpy(k_cache).to(self.device, q.dtype) if numpy_cache else k_cache
        vc = torch.from_numpy(v_cache).to(self.device, q.dtype) if numpy_cache else v_cache
        write_kv(k, v, kc, vc, slots)
        if numpy_cache:   # the reference's write_kv mutates the host cache
            k_cache[slots_np] = kc[slots].float().cpu().numpy()
            v_cache[slots_np] = vc[slots].float().cpu().numpy()
        tables = torch.as_tensor(np.asarray(layout.block_tables, dtype=np.int64),
                                 device=self.device)
        attended = paged_attention(q, kc, vc, tables, layout.context_lens, layout.query_lens,
                                   block_size)
        a = attended.reshape(-1, self.num_heads * self.config.head_dim).to(xt.dtype).contiguous()
        if comm is None:
            y = qlinear(a, self.o_proj)
        else:
            y = qlinear(a, self.o_proj, residual=xt, comm=comm)
        return y.cpu().numpy() if was_numpy else y


class ShardedMLP:
    """One rank's share of the SwiGLU MLP (ie/parallel/tensor_parallel.py:46-56):
    gate/up column shards (packed as row pairs so SiLU*up is fused into the
    GEMM epilogue) and the down row shard."""

    def __init__(self, block, shard: Shard, *, scheme: str = "int8", axis: int | None = 0,
                 device=None) -> None:
        if not all(isinstance(getattr(block, n), (QuantizedWeight, PackedWeight))
                   for n in MLP_PROJECTIONS):
            block = quantized_block(block, scheme, axis, names=MLP_PROJECTIONS)
        self._init(block.mlp_norm, block.gate_proj, block.up_proj, block.down_proj, shard,
                   float(block.config.norm_eps), device)

    @classmethod
    def from_weights(cls, norm, gate, up, down, shard: Shard, eps: float = 1e-6,
                     device=None) -> "ShardedMLP":
        """From the MLP's own tables: norm weight and the whole gate / up / down
        weights as ``QuantizedWeight`` or ``PackedWeight``."""
        self = cls.__new__(cls)
        self._init(norm, gate, up, down, shard, eps, device)
        return self

    def _init(self, norm, gate, up, down, shard, eps, device):
        torch = require_cuda()
        self.shard = shard
        self.eps = eps
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        self.norm = _f32(norm, self.device)
        g = _pack(split_output_dim(gate, shard), self.device)
        u = _pack(split_output_dim(up, shard), self.device)
        self.gate_up = PackedWeight.pair_gate_up(g, u)
        self.down = _pack(split_input_dim(down, shard), self.device)

    def forward(self, x, comm=None):
        """Partial ``(silu(n@g) * (n@u)) @ d`` (comm=None), or ``x + sum of partials``."""
        from .linear import fuse_norm_pays, qlinear

        xt, was_numpy = _to_device(x, self.device)
        if fuse_norm_pays(xt, self.gate_up):
            hidden = qlinear(xt, self.gate_up, silu_mul=True, norm_weight=self.norm,
                             norm_eps=self.eps)
        else:
            hidden = qlinear(rms_norm(xt, self.norm, self.eps), self.gate_up, silu_mul=True)
        if comm is None:
            y = qlinear(hidden, self.down, out_dtype=xt.dtype)
        else:
            y = qlinear(hidden, self.down, residual=xt, comm=comm, out_dtype=xt.dtype)
        return y.cpu().numpy() if was_numpy else y


class TensorParallelBlock:
    """ie/parallel/tensor_parallel.py:59-73: every rank's shards in this process,
    partials summed in rank order.  Each projection is quantized once, whole,
    and then sharded."""

    def __init__(self, block, world_size: int, *, scheme: str = "int8",
                 axis: int | None = 0, device=None) -> None:
        shards = [Shard(rank, world_size) for rank in range(world_size)]
        qblock = block if _is_quantized(block) else quantized_block(block, scheme, axis)
        self.attention = [ShardedAttention(qblock, s, device=device) for s in shards]
        self.mlp = [ShardedMLP(qblock, s, device=device) for s in shards]

    def forward(self, x, layout, k_caches, v_caches, cos, sin, block_size: int):
        partials = [rank.forward(x, layout, k_caches[i], v_caches[i], cos, sin, block_size)
                    for i, rank in enumerate(self.attention)]
        x = x + all_reduce(partials)
        partials = [rank.forward(x) for rank in self.mlp]
        return x + all_reduce(partials)
