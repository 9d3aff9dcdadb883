"""CPU oracle for the decoder around the quantized linear path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the ``ie_tpq`` package and
``libie_tpq.so``) imports, calls or links this module; only ``tests/`` and
``bench.py``'s CPU legs do.

A plain-NumPy restatement of the reference engine's random-init decoder
(kuluruvineeth/inference-engine, pure Python + NumPy), so that the GPU box,
which has no copy of the reference, can rebuild the same weights and the same
block outputs.  Every function names the reference file:line it restates.
Parity is PINNED by ``tests/test_oracle_golden.py`` against fixtures that
``tests/golden/make_golden.py`` and ``tests/golden/make_greedy.py`` produced by
running the reference itself (weight digests, a block forward, greedy tokens).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .tpq_oracle import rms_norm, silu


@dataclass
class Config:
    """ie/model/transformer.py:12-34 (the fields the forward uses)."""
    vocab_size: int = 256
    hidden_size: int = 64
    num_layers: int = 2
    num_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 16
    intermediate_size: int = 128
    max_position: int = 2048
    rope_base: float = 10000.0
    norm_eps: float = 1e-6
    rope_halved: bool = False


QWEN25_05B = Config(vocab_size=151936, hidden_size=896, num_layers=24, num_heads=14,
                    num_kv_heads=2, head_dim=64, intermediate_size=4864)


def rope_tables(max_position: int, head_dim: int, base: float = 10000.0):
    """ie/layers/functional.py:20-31."""
    exponents = np.arange(0, head_dim, 2, dtype=np.float32) / head_dim
    freqs = np.power(base, -exponents)
    angles = np.outer(np.arange(max_position, dtype=np.float32), freqs)
    return np.cos(angles), np.sin(angles)


def apply_rope(x, positions, cos_table, sin_table, halved: bool = False):
    """ie/layers/functional.py:34-61."""
    cos = cos_table[positions][:, None, :]
    sin = sin_table[positions][:, None, :]
    out = np.empty_like(x)
    if halved:
        half = x.shape[-1] // 2
        left, right = x[..., :half], x[..., half:]
        out[..., :half] = left * cos - right * sin
        out[..., half:] = right * cos + left * sin
    else:
        even, odd = x[..., 0::2], x[..., 1::2]
        out[..., 0::2] = even * cos - odd * sin
        out[..., 1::2] = even * sin + odd * cos
    return out


class Block:
    """ie/model/transformer.py:37-61: weights N(0, 1)/sqrt(hidden) in [in, out]
    layout, drawn in the order q, k, v, o, gate, up, down."""

    def __init__(self, config: Config, generator: np.random.Generator) -> None:
        self.config = config
        scale = 1.0 / np.sqrt(config.hidden_size)
        q_out = config.num_heads * config.head_dim
        kv_out = config.num_kv_heads * config.head_dim

        def normal(*shape):
            return (generator.standard_normal(shape) * scale).astype(np.float32)

        self.attn_norm = np.ones(config.hidden_size, dtype=np.float32)
        self.q_proj = normal(config.hidden_size, q_out)
        self.k_proj = normal(config.hidden_size, kv_out)
        self.v_proj = normal(config.hidden_size, kv_out)
        self.o_proj = normal(q_out, config.hidden_size)
        self.q_bias = np.zeros(q_out, dtype=np.float32)
        self.k_bias = np.zeros(kv_out, dtype=np.float32)
        self.v_bias = np.zeros(kv_out, dtype=np.float32)
        self.q_norm = None
        self.k_norm = None
        self.mlp_norm = np.ones(config.hidden_size, dtype=np.float32)
        self.gate_proj = normal(config.hidden_size, config.intermediate_size)
        self.up_proj = normal(config.hidden_size, config.intermediate_size)
        self.down_proj = normal(config.intermediate_size, config.hidden_size)


class Model:
    """ie/model/transformer.py:90-103: embedding, blocks, final norm, lm_head, rope tables."""

    def __init__(self, config: Config, seed: int = 0) -> None:
        self.config = config
        generator = np.random.default_rng(seed)
        scale = 1.0 / np.sqrt(config.hidden_size)
        self.embedding = (generator.standard_normal(
            (config.vocab_size, config.hidden_size)) * scale).astype(np.float32)
        self.blocks = [Block(config, generator) for _ in range(config.num_layers)]
        self.final_norm = np.ones(config.hidden_size, dtype=np.float32)
        self.lm_head = (generator.standard_normal(
            (config.hidden_size, config.vocab_size)) * scale).astype(np.float32)
        self.cos, self.sin = rope_tables(config.max_position, config.head_dim, config.rope_base)


def allocate_kv_cache(num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int):
    """ie/kernels/reference.py:36-39."""
    shape = (num_blocks * block_size, num_kv_heads, head_dim)
    return np.zeros(shape, np.float32), np.zeros(shape, np.float32)


def write_kv(k, v, k_cache, v_cache, slot_mapping) -> None:
    """ie/kernels/reference.py:42-49."""
    slots = np.asarray(slot_mapping, dtype=np.int64)
    k_cache[slots] = k
    v_cache[slots] = v


def _gather(cache, table, context_len: int, block_size: int):
    """ie/kernels/reference.py:52-62."""
    needed = (context_len + block_size - 1) // block_size
    slots = np.concatenate([np.arange(table[i] * block_size, (table[i] + 1) * block_size)
                            for i in range(needed)])
    return cache[slots[:context_len]]


def _dense_attention(q, k, v, query_offset: int):
    """ie/kernels/reference.py:20-33 (causal), with kv heads repeated (:12-17)."""
    query_len, heads, head_dim = q.shape
    if k.shape[1] != heads:
        k = np.repeat(k, heads // k.shape[1], axis=1)
        v = np.repeat(v, heads // v.shape[1], axis=1)
    scores = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(head_dim)
    rows = np.arange(query_len)[:, None] + query_offset
    cols = np.arange(k.shape[0])[None, :]
    scores = np.where(cols <= rows, scores, -np.inf)
    scores = scores - scores.max(axis=-1, keepdims=True)
    w = np.exp(scores)
    w = w / w.sum(axis=-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", w, v)


def paged_attention(q, k_cache, v_cache, block_tables, context_lens, query_lens, block_size):
    """ie/kernels/reference.py:65-80."""
    outs, start = [], 0
    for table, ctx, ql in zip(block_tables, context_lens, query_lens):
        k = _gather(k_cache, table, ctx, block_size)
        v = _gather(v_cache, table, ctx, block_size)
        outs.append(_dense_attention(q[start:start + ql], k, v, ctx - ql))
        start += ql
    return np.concatenate(outs, axis=0)


def block_forward(block, x, layout, k_cache, v_cache, cos, sin, block_size: int):
    """ie/model/transformer.py:63-87."""
    c = block.config
    normed = rms_norm(x, block.attn_norm, c.norm_eps)
    q = (normed @ block.q_proj + block.q_bias).reshape(-1, c.num_heads, c.head_dim)
    k = (normed @ block.k_proj + block.k_bias).reshape(-1, c.num_kv_heads, c.head_dim)
    v = (normed @ block.v_proj + block.v_bias).reshape(-1, c.num_kv_heads, c.head_dim)
    positions = np.asarray(layout.positions)
    q = apply_rope(q, positions, cos, sin, c.rope_halved)
    k = apply_rope(k, positions, cos, sin, c.rope_halved)
    write_kv(k, v, k_cache, v_cache, layout.slot_mapping)
    attended = paged_attention(q, k_cache, v_cache, layout.block_tables, layout.context_lens,
                               layout.query_lens, block_size)
    x = x + attended.reshape(-1, c.num_heads * c.head_dim) @ block.o_proj
    normed = rms_norm(x, block.mlp_norm, c.norm_eps)
    return x + (silu(normed @ block.gate_proj) * (normed @ block.up_proj)) @ block.down_proj


def fake_quantize_int8(model: Model) -> None:
    """ie/quant/model.py:42-52 with INT8 on axis 0: every projection replaced
    by its dequantized int8 weight, in place."""
    from .tpq_oracle import quantize_integer

    for block in model.blocks:
        for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                     "down_proj"):
            setattr(block, name, quantize_integer(getattr(block, name), 8, True, 0).dequantized())


def seeded_prompts(count: int, low: int, high: int, vocab: int, seed: int) -> list[list[int]]:
    """Prompt lengths uniform in [low, high], token ids uniform over the whole
    vocabulary (the workload of the Qwen-shaped config)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(low, high + 1, size=count)
    return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens]
