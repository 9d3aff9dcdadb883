"""A decoder's quantized tensor-parallel linear path, one rank's share.

Per layer (the order of TorchBlock.forward, ie/model/torch_transformer.py:31-63,
restricted to the linear path):

    h   = rms_norm(x)                      (attn_norm)
    qkv = h @ [Wq | Wk | Wv]_rank          column-parallel, head-sharded
    x   = x + all_reduce(a @ Wo_rank)      row-parallel, fused all-reduce + residual
    h   = rms_norm(x)                      (mlp_norm)
    u   = silu(h @ Wg_rank) * (h @ Wu_rank) column-parallel pair, fused SiLU*up
    x   = x + all_reduce(u @ Wd_rank)      row-parallel, fused all-reduce + residual

Attention sits between qkv and the o projection and is not part of this path;
``a`` is the q slice of the qkv output (the attention output has the q
projection's shape), so the stack streams exactly the layer's weights.

``capture()`` records one step as a CUDA graph; ``replay()`` launches it.  The
fused all-reduce keeps its epoch on the device, so replays stay paired
across ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import _lib
from .device import require_cuda
from .linear import fuse_norm_pays, qlinear
from .packed import PackedWeight, concat_rows, quantize_on_device
from .sharding import Shard
from .tensor_parallel import rms_norm


@dataclass
class DecoderShape:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    layers: int

    @property
    def q_out(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_out(self) -> int:
        return self.kv_heads * self.head_dim


LLAMA3_8B = DecoderShape(hidden=4096, heads=32, kv_heads=8, head_dim=128, intermediate=14336,
                         layers=32)
LLAMA3_70B = DecoderShape(hidden=8192, heads=64, kv_heads=8, head_dim=128, intermediate=28672,
                          layers=80)
QWEN25_05B = DecoderShape(hidden=896, heads=14, kv_heads=2, head_dim=64, intermediate=4864,
                          layers=24)


def layer_weight_bytes(shape: DecoderShape, scheme: str, world: int) -> dict[str, float]:
    """Algorithmic HBM bytes of one rank's packed weights per projection."""
    h, i = shape.hidden, shape.intermediate
    dims = {"qkv": (h, (shape.q_out + 2 * shape.kv_out) // world), "o": (shape.q_out // world, h),
            "gate_up": (h, 2 * i // world), "down": (i // world, h)}
    out = {}
    for name, (k, n) in dims.items():
        if scheme == "int4-g128":
            out[name] = k * n / 2 + (k // 128) * n * 4
        elif scheme == "int4":
            out[name] = k * n / 2 + 4 * k
        elif scheme == "fp8-native":   # per-N scales
            out[name] = k * n + 4 * n
        else:
            out[name] = k * n + 4 * k
    return out


def synthetic_layer(shape: DecoderShape, scheme: str, shard: Shard, seed: int,
                    std: float = 0.02) -> dict:
    """One layer's packed shards from N(0, std) f32 weights generated on the device
    (the whole weight, then this rank's slice, as the reference shards it)."""
    torch = require_cuda()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    h, i = shape.hidden, shape.intermediate

    def full(k, n):
        return torch.randn((k, n), generator=gen, device="cuda", dtype=torch.float32) * std

    def column(w, heads=None):
        sl = shard.slice_of(heads) if heads else shard.slice_of(w.shape[1])
        if heads:
            hd = w.shape[1] // heads
            sl = slice(sl.start * hd, sl.stop * hd)
        return quantize_on_device(w, scheme).slice_rows(sl.start, sl.stop)

    def row(w):
        sl = shard.slice_of(w.shape[0])
        return quantize_on_device(w, scheme).slice_k(sl.start, sl.stop)

    q = column(full(h, shape.q_out), shape.heads)
    k = column(full(h, shape.kv_out), shape.kv_heads)
    v = column(full(h, shape.kv_out), shape.kv_heads)
    o = row(full(shape.q_out, h))
    gate = column(full(h, i))
    up = column(full(h, i))
    down = row(full(i, h))
    layer = {"o": o, "gate_up": PackedWeight.pair_gate_up(gate, up), "down": down}
    if scheme == "int4-g128":
        layer["qkv"] = concat_rows([q, k, v])
    else:
        layer["q"], layer["k"], layer["v"] = q, k, v
    torch.cuda.empty_cache()
    return layer


class LinearStack:
    """The linear path of ``len(layers)`` decoder layers for one TP rank."""

    def __init__(self, shape: DecoderShape, layers: list[dict], batch: int, dtype=None,
                 comm=None, world: int = 1, fuse_norm: bool = True):
        torch = require_cuda()
        self.shape = shape
        self.layers = layers
        self.batch = batch
        self.dtype = dtype or torch.bfloat16
        self.comm = comm
        self.world = world
        h = shape.hidden
        self.norm = torch.ones(h, dtype=torch.float32, device="cuda")
        self.x_in = torch.zeros((batch, h), dtype=self.dtype, device="cuda")
        self.x_out = torch.zeros((batch, h), dtype=self.dtype, device="cuda")
        self.graph = None
        self.launches_per_step = 0
        # fold each rms_norm into the column-parallel GEMM that consumes it
        self.fuse_norm = fuse_norm

    def _row(self, a, w, residual):
        if self.comm is not None and self.world > 1:
            return qlinear(a, w, residual=residual, comm=self.comm)
        return qlinear(a, w, residual=residual)

    def _norm(self, x, w):
        """(input, norm weight) for the GEMM after a norm: x itself and the
        weight when the GEMM folds the norm in, else the normalised x."""
        if self.fuse_norm and fuse_norm_pays(x, w):
            return x, self.norm
        return rms_norm(x, self.norm), None

    def forward(self, x):
        """One decode step over all layers; returns the new hidden state."""
        q_cols = self.shape.q_out // self.world
        launches = 0
        for layer in self.layers:
            first = layer["qkv"] if "qkv" in layer else layer["q"]
            h, nw = self._norm(x, first)
            launches += nw is None
            if "qkv" in layer:
                qkv = qlinear(h, layer["qkv"], norm_weight=nw)
                a = qkv[:, :q_cols]
                launches += 1
            else:
                a = qlinear(h, layer["q"], norm_weight=nw)
                qlinear(h, layer["k"], norm_weight=nw)
                qlinear(h, layer["v"], norm_weight=nw)
                launches += 3
            x = self._row(a, layer["o"], x)
            h, nw = self._norm(x, layer["gate_up"])
            u = qlinear(h, layer["gate_up"], norm_weight=nw)
            x = self._row(u, layer["down"], x)
            launches += 3 + (nw is None)
        self.launches_per_step = launches
        return x

    def capture(self):
        """Record one step (x_in -> x_out) as a CUDA graph."""
        torch = require_cuda()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):   # warm up allocator pools outside the capture
                self.x_out.copy_(self.forward(self.x_in))
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.x_out.copy_(self.forward(self.x_in))
        self.graph = g
        return g

    def replay(self):
        self.graph.replay()

    def run_host(self, x_host, out_host):
        """End-to-end step through host buffers: H2D copy, the step, D2H copy."""
        self.x_in.copy_(x_host, non_blocking=True)
        self.graph.replay()
        out_host.copy_(self.x_out, non_blocking=True)


__all__ = ["DecoderShape", "LLAMA3_8B", "LLAMA3_70B", "QWEN25_05B", "LinearStack",
           "synthetic_layer", "layer_weight_bytes", "_lib"]
