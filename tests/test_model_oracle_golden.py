"""Pin the decoder oracle (oracle/model_oracle.py) to the reference engine:
weight initialisation, a block forward (dense and int8 fake-quantized) and the
seeded prompts, against tests/golden/golden_model.npz, which
tests/golden/make_model_golden.py produced by running the reference itself."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from oracle import model_oracle as mo
from tests.hashing import digest

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "golden_model.npz"
TINY = mo.Config(vocab_size=64, hidden_size=32, num_layers=1, num_heads=4, num_kv_heads=2,
                 head_dim=8, intermediate_size=64)


@pytest.fixture(scope="module")
def gm():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def tiny_layout(gm):
    pos = gm["tiny_positions"].tolist()
    return SimpleNamespace(positions=pos, slot_mapping=gm["tiny_slots"].tolist(),
                           block_tables=gm["tiny_tables"].tolist(), context_lens=[len(pos)],
                           query_lens=[len(pos)])


def test_tiny_model_weights_are_the_references_bitwise(gm):
    model = mo.Model(TINY, seed=3)
    assert np.array_equal(model.embedding, gm["tiny_embedding"])
    assert np.array_equal(model.lm_head, gm["tiny_lm_head"])
    for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
        assert np.array_equal(getattr(model.blocks[0], name), gm[f"tiny_{name}"]), name


@pytest.mark.parametrize("tag", ["dense", "int8"])
def test_block_forward_matches_the_reference(gm, tag):
    model = mo.Model(TINY, seed=3)
    if tag == "int8":
        mo.fake_quantize_int8(model)
    kc, vc = mo.allocate_kv_cache(64, 8, TINY.num_kv_heads, TINY.head_dim)
    lay = tiny_layout(gm)
    y = mo.block_forward(model.blocks[0], gm["tiny_x"], lay, kc, vc, model.cos, model.sin, 8)
    np.testing.assert_allclose(y, gm[f"tiny_block_out_{tag}"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(kc[np.asarray(lay.slot_mapping)], gm[f"tiny_kcache_{tag}"])


def test_qwen_shaped_init_digests(gm):
    """The first draws of the Qwen2.5-0.5B-shaped model (embedding, then block
    0's q projection) reproduce the reference's arrays bit for bit."""
    cfg = mo.QWEN25_05B
    gen = np.random.default_rng(0)
    scale = 1.0 / np.sqrt(cfg.hidden_size)
    emb = (gen.standard_normal((cfg.vocab_size, cfg.hidden_size)) * scale).astype(np.float32)
    assert digest(emb) == gm["qwen_digests"][0]
    del emb
    block = mo.Block(cfg, gen)
    assert digest(block.q_proj) == gm["qwen_digests"][2]


def test_seeded_prompts_are_the_fixtures(gm):
    prompts = mo.seeded_prompts(8, 128, 300, mo.QWEN25_05B.vocab_size, seed=2024)
    lens = gm["qwen_prompt_lens"]
    assert [len(p) for p in prompts] == lens.tolist()
    for i, p in enumerate(prompts):
        assert p == gm["qwen_prompts"][i, :lens[i]].tolist()
    assert gm["qwen_tokens"].shape == (8, 32)
