"""A decoder whose linear layers are this library's quantized tensor-parallel
shards, behind the reference engine's model protocol.

``QuantizedTransformer`` implements what ``Engine`` calls on a model
(ie/engine/engine.py:38-95, as ``TorchTransformer`` does in
ie/model/torch_transformer.py:82-140): ``allocate_caches``, ``uses_flash``,
``run``, ``forward``, ``logits_for_last_token_of_each``, ``logits_on_device``,
``sample``, plus ``config``, ``device``, ``dtype`` and ``graphs`` (so the
reference's ``DecodeGraphs`` can capture and replay its decode step).

One instance holds ONE tensor-parallel rank (``shard``); with one process per
GPU every rank builds its own instance from the same source model and steps the
same schedule, and the row-parallel o / down projections reduce across ranks
inside their GEMM epilogues through ``comm`` (ie/parallel/tensor_parallel.py:59-73
restated as SPMD).  Per layer (TorchBlock.forward, torch_transformer.py:31-63):

    q, k, v  = rms_norm(x) @ [Wq|Wk|Wv]_r (+ bias)   head-sharded, norm folded in
    q, k     = rope(q), rope(k); write_kv; attention over this rank's kv heads
    x        = x + all_reduce(attn @ Wo_r)            fused reduce + residual
    x        = x + all_reduce(silu(n @ Wg_r) * (n @ Wu_r) @ Wd_r)

The KV caches hold ``kv_heads / world`` heads per rank (tensor_parallel.py:76-79).
``lm_head`` is vocab-parallel: rank r holds columns ``[r V/w, (r+1) V/w)``;
``logits_on_device`` gathers the full row on every rank (each rank adds its
slice into a zeroed ``[B, V]`` buffer and the buffer is all-reduced: adding
zeros is exact, so this is a concatenation).  The lm_head is not quantized
unless ``quantize_lm_head`` (the reference's default, ie/quant/model.py:58-63);
the dense slice is a plain cuBLAS GEMM.  Sampling runs on the device
(torch_transformer.py:131-140); under TP the tokens of rank 0 are broadcast
the same way, so every rank continues with identical tokens.
"""
from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import numpy as np

from .attention import (FLASH, PAGED_FLASH_BLOCK, allocate_kv_cache, apply_rope, flash_decode,
                        flash_prefill, paged_attention, rope_write_kv, write_kv)
from .device import require_cuda
from .sharding import Shard
from .tensor_parallel import (ShardedAttention, ShardedMLP, kv_heads_per_rank, quantized_block,
                              rms_norm)


@dataclass
class DecoderConfig:
    """The model fields the forward uses (ie/model/transformer.py:12-34)."""
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    max_position: int = 4096
    rope_base: float = 500000.0
    norm_eps: float = 1e-5
    rope_halved: bool = False


LLAMA3_8B_CONFIG = DecoderConfig(vocab_size=128256, hidden_size=4096, num_layers=32,
                                 num_heads=32, num_kv_heads=8, head_dim=128,
                                 intermediate_size=14336)
LLAMA3_70B_CONFIG = DecoderConfig(vocab_size=128256, hidden_size=8192, num_layers=80,
                                  num_heads=64, num_kv_heads=8, head_dim=128,
                                  intermediate_size=28672, max_position=8192)


def rope_tables_on_device(max_position: int, head_dim: int, base: float, device):
    """cos / sin tables (ie/layers/functional.py:20-31) as f32 device tensors."""
    torch = require_cuda()
    exps = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim
    freqs = torch.pow(torch.tensor(base, dtype=torch.float32, device=device), -exps)
    angles = torch.outer(torch.arange(max_position, dtype=torch.float32, device=device), freqs)
    return torch.cos(angles), torch.sin(angles)


def synthetic_source(config: DecoderConfig, scheme: str, seed: int = 0, std: float = 0.02,
                     dtype=None, device="cuda"):
    """A random-init decoder with the reference Transformer's layout (blocks of
    seven ``[K, N]`` projections, norms, embedding, lm_head, RoPE tables), drawn
    N(0, std) on the device and quantized there with the reference's tables
    (``quantize_on_device``): no host copy of the f32 weights, which for a
    Llama-3-8B shape would be 32 GB.  ``blocks`` yields one block at a time, so
    a tensor-parallel rank holds one full block plus its shards.  Norm weights
    are ones."""
    torch = require_cuda()
    from .packed import quantize_on_device

    dtype = dtype or torch.bfloat16
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    h, i = config.hidden_size, config.intermediate_size
    q_out, kv_out = config.num_heads * config.head_dim, config.num_kv_heads * config.head_dim

    def quant(k, n):
        w = torch.randn((k, n), generator=gen, device=device, dtype=torch.float32) * std
        return quantize_on_device(w, scheme)

    def blocks():   # one block at a time: a consumer keeps only its shards
        for _ in range(config.num_layers):
            yield SimpleNamespace(
                config=config, q_proj=quant(h, q_out), k_proj=quant(h, kv_out),
                v_proj=quant(h, kv_out), o_proj=quant(q_out, h), gate_proj=quant(h, i),
                up_proj=quant(h, i), down_proj=quant(i, h),
                attn_norm=torch.ones(h, dtype=torch.float32, device=device),
                mlp_norm=torch.ones(h, dtype=torch.float32, device=device),
                q_bias=None, k_bias=None, v_bias=None, q_norm=None, k_norm=None)
            torch.cuda.empty_cache()

    rnd = lambda *shape: (torch.randn(shape, generator=gen, device=device,
                                      dtype=torch.float32) * std).to(dtype)
    cos, sin = rope_tables_on_device(config.max_position, config.head_dim, config.rope_base,
                                     device)
    return SimpleNamespace(config=config, blocks=blocks(), embedding=rnd(config.vocab_size, h),
                           final_norm=torch.ones(h, dtype=torch.float32, device=device),
                           lm_head=rnd(h, config.vocab_size), cos=cos, sin=sin)


class QuantizedTransformer:
    def __init__(self, source, *, scheme: str = "int8", axis: int | None = 0,
                 shard: Shard | None = None, comm=None, device="cuda", dtype=None,
                 quantize_lm_head: bool = False) -> None:
        torch = require_cuda()
        self.config = source.config
        self.shard = shard or Shard(0, 1)
        self.world = self.shard.world_size
        self.comm = comm
        if self.world > 1 and comm is None:
            raise ValueError("a tensor-parallel rank needs a Communicator (comm=)")
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype or torch.float16
        self.scheme = scheme
        kv_heads_per_rank(self.config, self.world)   # raises like the reference
        def take(w, dt=None):
            t = w if isinstance(w, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(w))
            return t.to(device=self.device, dtype=dt or self.dtype).contiguous()

        self.embedding = take(source.embedding)
        self.attn, self.mlp = [], []
        # "fp8-native": fp8 weights with per-N scales whose activations are
        # quantized per token to e4m3 and contracted on the tensor cores
        native = scheme == "fp8-native"
        qscheme, qaxis = ("fp8", 1) if native else (scheme, axis)
        for block in source.blocks:
            qb = quantized_block(block, qscheme, qaxis)
            attn = ShardedAttention(qb, self.shard, device=self.device)
            mlp = ShardedMLP(qb, self.shard, device=self.device)
            if native:
                from . import _lib

                for w in (attn.qkv, attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj,
                          mlp.gate_up, mlp.down):
                    if w is not None:
                        w.act_quant = _lib.IE_ACT_FP8_TOKEN
            self.attn.append(attn)
            self.mlp.append(mlp)
            torch.cuda.empty_cache()
        self.final_norm = take(source.final_norm, torch.float32)
        vocab = self.config.vocab_size
        cols = self.shard.slice_of(vocab)
        self.vocab_slice = cols
        self.lm_head_packed = None
        if quantize_lm_head:
            from .sharding import split_output_dim

            if isinstance(source.lm_head, torch.Tensor):
                from .packed import quantize_on_device

                q = quantize_on_device(source.lm_head.to(self.device, torch.float32).contiguous(),
                                       scheme, axis)
                self.lm_head_packed = split_output_dim(q, self.shard)
            else:
                from .quant_model import quantize_for_device

                q = quantize_for_device(np.asarray(source.lm_head, np.float32), scheme, axis)
                self.lm_head_packed = split_output_dim(q, self.shard).packed(self.device)
            self.lm_head = None
        elif isinstance(source.lm_head, torch.Tensor):
            self.lm_head = take(source.lm_head[:, cols])
        else:
            self.lm_head = take(np.asarray(source.lm_head)[:, cols])
        self.cos = take(source.cos, torch.float32)
        self.sin = take(source.sin, torch.float32)
        self.graphs = None
        self.num_heads = self.config.num_heads // self.world
        self.num_kv_heads = self.config.num_kv_heads // self.world

    # ---- engine protocol ------------------------------------------------------
    def allocate_caches(self, num_blocks: int, block_size: int):
        """ie/model/torch_transformer.py:82-86 with this rank's kv heads."""
        pairs = [allocate_kv_cache(num_blocks, block_size, self.num_kv_heads,
                                   self.config.head_dim, self.device, self.dtype)
                 for _ in range(self.config.num_layers)]
        return [p[0] for p in pairs], [p[1] for p in pairs]

    @property
    def uses_flash(self) -> bool:
        torch = require_cuda()
        return FLASH and self.dtype in (torch.float16, torch.bfloat16)

    def _reduce(self):
        return self.comm if self.world > 1 else None

    def _layer(self, i, x, positions, block_tables, plan, layout, k_cache, v_cache,
               block_size):
        from .linear import qlinear

        attn, mlp = self.attn[i], self.mlp[i]
        # A prefill of fresh prompts attends over its own k and v (not the
        # cache) and needs them as tensors; every other step reads the cache.
        needs_kv = plan["flash"] and layout.is_prefill and plan["paged_tables"] is None
        qkv = None if needs_kv else attn.fused_qkv(x)
        if qkv is not None:   # RoPE of q and k and the cache write in one launch
            q = rope_write_kv(qkv, attn.num_heads, attn.num_kv_heads, self.config.head_dim,
                              positions, self.cos, self.sin, plan["slots"], k_cache, v_cache,
                              attn.rope_halved)
            k = v = None
        else:
            q, k, v = attn.project_qkv(x)
            q = apply_rope(q, positions, self.cos, self.sin, attn.rope_halved)
            k = apply_rope(k, positions, self.cos, self.sin, attn.rope_halved)
            write_kv(k, v, k_cache, v_cache, plan["slots"])
        if plan["flash"]:
            if layout.is_prefill:
                attended = flash_prefill(q, k, v, k_cache, v_cache, plan["cu_q"], plan["cu_k"],
                                         layout.max_query_len, layout.max_context_len,
                                         plan["paged_tables"], block_size, plan["scale"])
            else:
                tables = plan.get("tables32")
                attended = flash_decode(q, k_cache, v_cache,
                                        tables if tables is not None else block_tables.int(),
                                        plan["context_lens"], block_size, plan["scale"])
        else:
            attended = paged_attention(q, k_cache, v_cache, block_tables, layout.context_lens,
                                       layout.query_lens, block_size)
        a = attended.reshape(-1, self.num_heads * self.config.head_dim).to(x.dtype).contiguous()
        x = qlinear(a, attn.o_proj, residual=x, comm=self._reduce())
        from .linear import fuse_norm_pays

        if fuse_norm_pays(x, mlp.gate_up):
            hidden = qlinear(x, mlp.gate_up, silu_mul=True, norm_weight=mlp.norm,
                             norm_eps=mlp.eps)
        else:
            hidden = qlinear(rms_norm(x, mlp.norm, mlp.eps), mlp.gate_up, silu_mul=True)
        return qlinear(hidden, mlp.down, residual=x, comm=self._reduce(), out_dtype=x.dtype)

    def run(self, tokens, positions, block_tables, plan, layout, k_caches, v_caches,
            block_size: int):
        """ie/model/torch_transformer.py:92-98."""
        x = self.embedding.index_select(0, tokens)
        for i in range(len(self.attn)):
            x = self._layer(i, x, positions, block_tables, plan, layout, k_caches[i],
                            v_caches[i], block_size)
        return rms_norm(x, self.final_norm, self.config.norm_eps)

    def forward(self, layout, k_caches, v_caches, block_size: int):
        """ie/model/torch_transformer.py:100-122."""
        torch = require_cuda()
        if self.graphs is not None and self.graphs.can_replay(layout):
            return self.graphs.replay(layout, k_caches, v_caches)
        as_tensor = lambda values, dtype=torch.long: torch.as_tensor(
            np.asarray(values), device=self.device, dtype=dtype)
        tokens = as_tensor(layout.token_ids)
        positions = as_tensor(layout.positions)
        block_tables = as_tensor(layout.block_tables)
        # flash-attn's paged kernels (decode, and prefill over cached context)
        # take only page sizes that are multiples of PAGED_FLASH_BLOCK; other
        # block sizes run those steps on the torch paged-attention path.  A
        # prefill of fresh prompts reads no cache and always takes flash.
        paged = (not layout.is_prefill) or layout.max_context_len > layout.max_query_len
        use_flash = self.uses_flash and (not paged or block_size % PAGED_FLASH_BLOCK == 0)
        plan = {
            "flash": use_flash,
            "scale": self.config.head_dim ** -0.5,
            "slots": as_tensor(layout.slot_mapping),
            "cu_q": as_tensor(layout.cu_seqlens_q, torch.int32) if use_flash else None,
            "cu_k": as_tensor(layout.cu_seqlens_k, torch.int32) if use_flash else None,
            "context_lens": as_tensor(layout.context_lens, torch.int32) if use_flash else None,
            "paged_tables": (block_tables.to(torch.int32)
                             if use_flash and layout.max_context_len > layout.max_query_len
                             else None),
            "tables32": (block_tables.to(torch.int32)
                         if use_flash and not layout.is_prefill else None),
        }
        return self.run(tokens, positions, block_tables, plan, layout, k_caches, v_caches,
                        block_size)

    def logits_on_device(self, hidden, query_lens) -> "torch.Tensor":
        """Full-vocabulary logits of each sequence's last token, on every rank."""
        torch = require_cuda()
        ends = torch.as_tensor(np.cumsum(query_lens) - 1, device=self.device, dtype=torch.long)
        h = hidden.index_select(0, ends)
        if self.lm_head_packed is not None:
            from .linear import qlinear

            local = qlinear(h.contiguous(), self.lm_head_packed, out_dtype=torch.float32)
        else:
            local = (h @ self.lm_head).float()
        if self.world == 1:
            return local
        full = torch.zeros((h.shape[0], self.config.vocab_size), dtype=torch.float32,
                           device=self.device)
        full[:, self.vocab_slice] = local
        return self.comm.all_reduce(full)

    def greedy_on_device(self, hidden) -> "torch.Tensor":
        """Argmax token of every row of ``hidden`` as a device tensor, without
        gathering full-vocabulary logits: each rank takes the first maximum of
        its vocabulary slice, and the ranks' (value, index) pairs are summed
        into a zeroed [world, 2, rows] buffer (a concatenation); the first
        rank holding the largest value wins, which is the first maximum of
        the full row (torch_transformer.py:131-140 at temperature 0)."""
        torch = require_cuda()
        if self.lm_head_packed is not None:
            from .linear import qlinear

            local = qlinear(hidden.contiguous(), self.lm_head_packed, out_dtype=torch.float32)
        else:
            local = (hidden @ self.lm_head).float()
        idx = local.argmax(dim=-1)
        if self.world == 1:
            return idx
        val = local.gather(1, idx[:, None]).squeeze(1)
        buf = torch.zeros((self.world, 2, hidden.shape[0]), dtype=torch.float32,
                          device=self.device)
        buf[self.shard.rank, 0] = val
        buf[self.shard.rank, 1] = (idx + self.vocab_slice.start).float()
        both = self.comm.all_reduce(buf)
        best = both[:, 0].argmax(dim=0)
        return both[:, 1].gather(0, best[None]).squeeze(0).long()

    def logits_for_last_token_of_each(self, hidden, query_lens) -> np.ndarray:
        return self.logits_on_device(hidden, query_lens).float().cpu().numpy()

    def sample(self, hidden, query_lens, temperatures) -> list[int]:
        """ie/model/torch_transformer.py:131-140: argmax for temperature 0, else
        the exponential race over softmax(logits / T); rank 0's choice wins."""
        torch = require_cuda()
        logits = self.logits_on_device(hidden, query_lens)
        temps = torch.as_tensor(np.asarray(temperatures, dtype=np.float32), device=self.device)
        greedy = temps <= 0.0
        safe = torch.where(greedy, torch.ones_like(temps), temps).unsqueeze(1)
        probs = torch.softmax(logits / safe, dim=-1)
        race = torch.empty_like(probs).exponential_(1.0).clamp_min(1e-10)
        sampled = (probs / race).argmax(dim=-1)
        chosen = torch.where(greedy, logits.argmax(dim=-1), sampled)
        if self.world > 1 and not bool(greedy.all()):
            mine = chosen.to(torch.float32) if self.shard.rank == 0 else torch.zeros_like(
                chosen, dtype=torch.float32)
            chosen = self.comm.all_reduce(mine).round().long()
        return chosen.tolist()
