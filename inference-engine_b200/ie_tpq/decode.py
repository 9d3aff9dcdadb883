"""A fixed-batch greedy decode driver for the model protocol.

The reference drives a model through ``Engine.step()`` (scheduler, block
manager, ``build_layout``: ie/engine/engine.py:79-95, ie/core/layout.py:67-93).
That control plane is not part of this library.  This module is the minimal
stand-in used by the tests and the benchmark: every sequence of one batch gets
a contiguous run of KV blocks up front, the prompts are prefilled together,
and then each step decodes one token per sequence with greedy sampling.  The
layouts it builds carry the same fields as the reference's ``BatchLayout``,
so any model that implements the protocol (``QuantizedTransformer``, or the
reference's own models) runs under it.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Layout:
    """Field-for-field the reference's BatchLayout (ie/core/layout.py:10-45)."""
    token_ids: list[int]
    positions: list[int]
    slot_mapping: list[int]
    context_lens: list[int]
    query_lens: list[int]
    block_tables: list[list[int]]
    is_prefill: bool

    @property
    def num_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def cu_seqlens_q(self) -> list[int]:
        return [0] + list(np.cumsum(self.query_lens, dtype=np.int64).tolist())

    @property
    def cu_seqlens_k(self) -> list[int]:
        return [0] + list(np.cumsum(self.context_lens, dtype=np.int64).tolist())

    @property
    def max_query_len(self) -> int:
        return max(self.query_lens, default=0)

    @property
    def max_context_len(self) -> int:
        return max(self.context_lens, default=0)


class FixedBatch:
    """KV block tables for a fixed set of sequences: sequence i owns blocks
    ``[i*per, (i+1)*per)``."""

    def __init__(self, prompts: list[list[int]], max_new_tokens: int, block_size: int):
        self.block_size = block_size
        longest = max(len(p) for p in prompts) + max_new_tokens
        self.per = (longest + block_size - 1) // block_size
        self.tables = [list(range(i * self.per, (i + 1) * self.per)) for i in range(len(prompts))]
        self.num_blocks = self.per * len(prompts)
        self.tokens = [list(p) for p in prompts]

    def slot(self, seq: int, pos: int) -> int:
        return self.tables[seq][pos // self.block_size] * self.block_size + pos % self.block_size

    def prefill_layout(self, seqs=None) -> Layout:
        seqs = range(len(self.tokens)) if seqs is None else seqs
        ids, pos, slots, ctx, ql, tables = [], [], [], [], [], []
        for s in seqs:
            n = len(self.tokens[s])
            ids += self.tokens[s]
            pos += list(range(n))
            slots += [self.slot(s, p) for p in range(n)]
            ctx.append(n)
            ql.append(n)
            tables.append(self.tables[s])
        return Layout(ids, pos, slots, ctx, ql, tables, True)

    def decode_layout(self) -> Layout:
        ids, pos, slots, ctx = [], [], [], []
        for s, toks in enumerate(self.tokens):
            p = len(toks) - 1
            ids.append(toks[-1])
            pos.append(p)
            slots.append(self.slot(s, p))
            ctx.append(p + 1)
        return Layout(ids, pos, slots, ctx, [1] * len(self.tokens), list(self.tables), False)


def greedy_generate(model, prompts: list[list[int]], max_new_tokens: int, block_size: int = 16,
                    on_step=None) -> list[list[int]]:
    """Greedy tokens of every prompt (temperature 0), one prefill then one
    decode step per new token.  ``on_step(kind, layout)`` is called after each
    step (for timing)."""
    batch = FixedBatch(prompts, max_new_tokens, block_size)
    k_caches, v_caches = model.allocate_caches(batch.num_blocks, block_size)
    zeros = np.zeros(len(prompts), dtype=np.float32)
    layout = batch.prefill_layout()
    hidden = model.forward(layout, k_caches, v_caches, block_size)
    out = [[] for _ in prompts]
    for step in range(max_new_tokens):
        toks = model.sample(hidden, layout.query_lens, zeros)
        for s, t in enumerate(toks):
            out[s].append(int(t))
            batch.tokens[s].append(int(t))
        if on_step is not None:
            on_step("prefill" if step == 0 else "decode", layout)
        if step + 1 == max_new_tokens:
            break
        layout = batch.decode_layout()
        hidden = model.forward(layout, k_caches, v_caches, block_size)
    return out


def teacher_forced_predictions(model, sequences: list[list[int]], first: list[int],
                               block_size: int = 16):
    """Greedy predictions along known sequences: for sequence s, the argmax and
    the top-two logit gap at positions ``first[s] - 1 .. len - 2`` (row t
    predicts token t + 1), each sequence run as one prefill."""
    import torch

    batch = FixedBatch(sequences, 0, block_size)
    k_caches, v_caches = model.allocate_caches(batch.num_blocks, block_size)
    preds, gaps = [], []
    for s in range(len(sequences)):
        layout = batch.prefill_layout([s])
        hidden = model.forward(layout, k_caches, v_caches, block_size)
        rows = hidden[first[s] - 1:len(sequences[s]) - 1]
        logits = model.logits_on_device(rows.contiguous(), [1] * rows.shape[0])
        top = torch.topk(logits.float(), 2, dim=-1)
        preds.append(top.indices[:, 0].cpu().numpy())
        gaps.append((top.values[:, 0] - top.values[:, 1]).cpu().numpy())
    return preds, gaps
