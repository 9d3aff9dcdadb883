"""Generate the fixtures that pin the decoder oracle (oracle/model_oracle.py)
and record the reference engine's greedy tokens.

Run from the repository root where the reference engine
(kuluruvineeth/inference-engine, pure Python) is importable:

    IE_REFERENCE=/path/to/inference-engine python tests/golden/make_model_golden.py

Writes ``tests/golden/golden_model.npz``:

  * ``tiny_*`` -- a small random-init ``Transformer`` (the configuration of the
    reference's tests/test_tensor_parallel.py:20-21) and one block forward
    over a 12-token prefill with real RoPE tables, both with the dense f32
    weights and after int8 fake quantization (ie/quant/model.py:42-65);
  * ``qwen_*`` -- for the Qwen2.5-0.5B-shaped configuration (24 layers, hidden
    896, 14/2 heads, head_dim 64, MLP 4864, vocab 151936): digests of its
    seeded weights, 8 seeded prompts (lengths uniform in [128, 300], ids over
    the whole vocabulary), the 32 greedy tokens the reference ``Engine``
    generates for each of them after int8 fake quantization, and the top-two
    logit gap at every generated position (from one teacher-forced forward of
    the finished sequences), which tells a tie from a divergence.

The GPU box never runs this script; the tests read only its output.
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def digest(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def main() -> None:
    ref_root = os.environ.get("IE_REFERENCE")
    if not ref_root:
        raise SystemExit("set IE_REFERENCE to the reference engine's source tree")
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(REPO))

    from ie.core.block_manager import BlockManager
    from ie.core.layout import BatchLayout, build_layout
    from ie.core.scheduler import Scheduler
    from ie.core.sequence import Sequence
    from ie.engine.engine import Engine, EngineConfig
    from ie.kernels.reference import allocate_kv_cache
    from ie.model.transformer import ModelConfig, Transformer
    from ie.quant.formats import INT8
    from ie.quant.model import quantize_transformer

    from oracle.model_oracle import seeded_prompts

    out: dict[str, np.ndarray] = {}

    # --- tiny model: init and one block forward -------------------------------
    tiny = ModelConfig(vocab_size=64, hidden_size=32, num_layers=1, num_heads=4, num_kv_heads=2,
                       head_dim=8, intermediate_size=64)
    model = Transformer(tiny, seed=3)
    out["tiny_embedding"] = model.embedding
    out["tiny_lm_head"] = model.lm_head
    blk = model.blocks[0]
    for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
        out[f"tiny_{name}"] = getattr(blk, name)
    bs = 8
    manager = BlockManager(num_blocks=64, block_size=bs)
    sched = Scheduler(manager, max_batch_tokens=128)
    sched.add(Sequence(list(range(12)), block_size=bs))
    layout = build_layout(sched.schedule(), bs)
    out["tiny_positions"] = np.asarray(layout.positions)
    out["tiny_slots"] = np.asarray(layout.slot_mapping)
    out["tiny_tables"] = np.asarray(layout.block_tables)
    x = np.random.default_rng(7).standard_normal((layout.num_tokens, 32)).astype(np.float32)
    out["tiny_x"] = x
    for tag in ("dense", "int8"):
        if tag == "int8":
            quantize_transformer(model, INT8)
        kc, vc = allocate_kv_cache(64, bs, tiny.num_kv_heads, tiny.head_dim)
        out[f"tiny_block_out_{tag}"] = blk.forward(x, layout, kc, vc, model.cos, model.sin, bs)
        out[f"tiny_kcache_{tag}"] = kc[np.asarray(layout.slot_mapping)]

    # --- Qwen-shaped model: weight digests, greedy tokens, logit gaps ----------
    qcfg = ModelConfig(vocab_size=151936, hidden_size=896, num_layers=24, num_heads=14,
                       num_kv_heads=2, head_dim=64, intermediate_size=4864)
    qmodel = Transformer(qcfg, seed=0)
    digests = [digest(qmodel.embedding), digest(qmodel.lm_head),
               digest(qmodel.blocks[0].q_proj), digest(qmodel.blocks[23].down_proj)]
    out["qwen_digests"] = np.array(digests)
    quantize_transformer(qmodel, INT8)
    out["qwen_int8_digests"] = np.array([digest(qmodel.blocks[0].q_proj),
                                         digest(qmodel.blocks[23].down_proj)])
    prompts = seeded_prompts(8, 128, 300, qcfg.vocab_size, seed=2024)
    new_tokens = 32
    engine = Engine(qmodel, EngineConfig(block_size=16, num_blocks=1024,
                                         max_batch_tokens=4096, seed=0))
    gen = engine.generate(prompts, max_new_tokens=new_tokens, temperature=0.0)
    lens = np.array([len(p) for p in prompts])
    flat = np.zeros((len(prompts), int(lens.max())), dtype=np.int64)
    for i, p in enumerate(prompts):
        flat[i, :len(p)] = p
    out["qwen_prompt_lens"] = lens
    out["qwen_prompts"] = flat
    out["qwen_tokens"] = np.array(gen, dtype=np.int64)
    gaps = np.zeros((len(prompts), new_tokens), dtype=np.float32)
    for i, (p, g) in enumerate(zip(prompts, gen)):
        seq = list(p) + list(g)
        n = len(seq) - 1            # positions whose next token is known
        blocks = list(range((len(seq) + 15) // 16))
        lay = BatchLayout(token_ids=seq[:n], positions=list(range(n)),
                          slot_mapping=[blocks[t // 16] * 16 + t % 16 for t in range(n)],
                          context_lens=[n], query_lens=[n], block_tables=[blocks],
                          is_prefill=True)
        caches = [allocate_kv_cache(len(blocks), 16, qcfg.num_kv_heads, qcfg.head_dim)
                  for _ in range(qcfg.num_layers)]
        hidden = qmodel.forward(lay, [c[0] for c in caches], [c[1] for c in caches], 16)
        logits = hidden[len(p) - 1:] @ qmodel.lm_head
        top = np.sort(logits, axis=-1)[:, -2:]
        assert np.array_equal(np.argmax(logits, axis=-1), np.asarray(g)), "teacher-forced argmax"
        gaps[i] = top[:, 1] - top[:, 0]
    out["qwen_gaps"] = gaps
    np.savez_compressed(HERE / "golden_model.npz", **out)
    print(f"wrote {len(out)} arrays; min gap {gaps.min():.4g}")


if __name__ == "__main__":
    main()
