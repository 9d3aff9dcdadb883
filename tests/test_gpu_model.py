"""Parity of the tensor-parallel block and of the Engine-protocol model against
the reference, through the quantized kernels.

* ``TensorParallelBlock(block, world_size)`` / ``ShardedMLP(block, shard)`` /
  ``ShardedAttention(block, shard)`` -- the reference's constructors
  (ie/parallel/tensor_parallel.py:12-73) -- on the reference's own tiny block
  with int8 weights: NumPy f32 inputs run the f32 weight-streaming kernel and
  are held to 1e-4 against the reference's fake-quantized block output
  (tests/golden/golden_model.npz, produced by the reference); torch f16 inputs
  take the tensor-core kernel and are held to rtol 2e-2 / atol 2e-2 (the
  block carries f16 rounding of q, k, v, the attention output and the
  residual stream, beyond the linear layers' own rtol 2e-2 / atol 2e-3).
* ``QuantizedTransformer`` on the Qwen2.5-0.5B-shaped config (24 layers, int8
  per-channel) against the 32 greedy tokens the reference ``Engine`` produced
  for 8 seeded prompts.  With f32 activations every token must match.  With
  f16 activations the model is run teacher-forced along the reference's
  sequences: every prediction whose reference top-two logit gap exceeds 0.05
  must match, and free-running generation may first diverge only at such a
  near-tie (the reference's own tests assert exactness only in f32,
  tests/test_torch_backend.py:23-30)."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from ie_tpq.decode import greedy_generate, teacher_forced_predictions
from ie_tpq.model import QuantizedTransformer
from ie_tpq.sharding import Shard
from ie_tpq.tensor_parallel import ShardedAttention, ShardedMLP, TensorParallelBlock
from oracle import model_oracle as mo
from oracle import tpq_oracle as o

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "golden_model.npz"
TINY = mo.Config(vocab_size=64, hidden_size=32, num_layers=1, num_heads=4, num_kv_heads=2,
                 head_dim=8, intermediate_size=64)
TIE_GAP = 0.05


@pytest.fixture(scope="module")
def gm():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def tiny_layout(gm):
    pos = gm["tiny_positions"].tolist()
    return SimpleNamespace(positions=pos, slot_mapping=gm["tiny_slots"].tolist(),
                           block_tables=gm["tiny_tables"].tolist(), context_lens=[len(pos)],
                           query_lens=[len(pos)])


@pytest.mark.parametrize("world", [1, 2])
def test_tp_block_matches_the_reference_block(gm, world):
    model = mo.Model(TINY, seed=3)
    block = model.blocks[0]
    tp = TensorParallelBlock(block, world, scheme="int8")
    caches = [mo.allocate_kv_cache(64, 8, TINY.num_kv_heads // world, TINY.head_dim)
              for _ in range(world)]
    lay = tiny_layout(gm)
    y = tp.forward(gm["tiny_x"], lay, [c[0] for c in caches], [c[1] for c in caches],
                   model.cos, model.sin, 8)
    assert isinstance(y, np.ndarray)
    np.testing.assert_allclose(y, gm["tiny_block_out_int8"], rtol=1e-4, atol=1e-4)
    # each rank's cache holds its kv heads, written in place like the reference
    slots = np.asarray(lay.slot_mapping)
    k_all = np.concatenate([c[0][slots] for c in caches], axis=1)
    np.testing.assert_allclose(k_all, gm["tiny_kcache_int8"], rtol=1e-4, atol=1e-5)


def test_tp_block_f16_on_the_tensor_cores(gm):
    model = mo.Model(TINY, seed=3)
    tp = TensorParallelBlock(model.blocks[0], 2, scheme="int8")
    caches = [mo.allocate_kv_cache(64, 8, 1, TINY.head_dim) for _ in range(2)]
    kc = [torch.from_numpy(c[0]).cuda().half() for c in caches]
    vc = [torch.from_numpy(c[1]).cuda().half() for c in caches]
    x = torch.from_numpy(gm["tiny_x"]).cuda().half()
    y = tp.forward(x, tiny_layout(gm), kc, vc, model.cos, model.sin, 8)
    assert y.dtype == torch.float16
    np.testing.assert_allclose(y.float().cpu().numpy(), gm["tiny_block_out_int8"],
                               rtol=2e-2, atol=2e-2)


def test_each_rank_holds_its_fraction_of_the_weights():
    """tests/test_tensor_parallel.py:108-115 on the packed shards."""
    model = mo.Model(TINY, seed=4)
    tp = TensorParallelBlock(model.blocks[0], 2, scheme="int8")
    per_rank = [a.q_proj.codes.numel() + a.o_proj.codes.numel() for a in tp.attention]
    per_rank_mlp = [m.gate_up.codes.numel() + m.down.codes.numel() for m in tp.mlp]
    blk = model.blocks[0]
    whole = blk.q_proj.size + blk.o_proj.size
    whole_mlp = blk.gate_proj.size + blk.up_proj.size + blk.down_proj.size
    assert per_rank[0] * 2 == whole and per_rank[1] == per_rank[0]
    assert per_rank_mlp[0] * 2 == whole_mlp


@pytest.mark.parametrize("world", [1, 2, 4])
def test_sharded_mlp_takes_the_block(world):
    """ShardedMLP(block, shard) partials, summed in rank order, against the
    oracle's TP MLP on the fake-quantized weights (config 1's shapes)."""
    x, norm, gate, up, down = o.config1_inputs()
    blk = SimpleNamespace(config=SimpleNamespace(norm_eps=1e-6), mlp_norm=norm, gate_proj=gate,
                          up_proj=up, down_proj=down)
    xt = torch.from_numpy(x).cuda()
    parts = [ShardedMLP(blk, Shard(r, world), scheme="int8").forward(xt) for r in range(world)]
    got = (xt + sum(parts[1:], parts[0].clone())).cpu().numpy()
    deq = {n: o.quantize_integer(w, 8, True, 0).dequantized()
           for n, w in (("g", gate), ("u", up), ("d", down))}
    want = o.tp_mlp(x, norm, deq["g"], deq["u"], deq["d"], world)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_sharded_attention_shards_biases_with_their_heads():
    model = mo.Model(TINY, seed=5)
    blk = model.blocks[0]
    blk.q_bias = np.arange(blk.q_bias.size, dtype=np.float32)
    att = [ShardedAttention(blk, Shard(r, 2), scheme="int8") for r in range(2)]
    half = blk.q_bias.size // 2
    assert np.array_equal(att[1].q_bias.cpu().numpy(), blk.q_bias[half:])
    assert att[0].num_heads == 2 and att[0].num_kv_heads == 1


# ---------------------------------------------------------------------------
# the Engine-protocol model: greedy tokens of the Qwen2.5-0.5B-shaped config
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def qwen_source():
    return mo.Model(mo.QWEN25_05B, seed=0)


def prompts_of(gm):
    lens = gm["qwen_prompt_lens"]
    return [gm["qwen_prompts"][i, :lens[i]].tolist() for i in range(len(lens))]


def first_divergence(got, want):
    for j, (a, b) in enumerate(zip(got, want)):
        if a != b:
            return j
    return None


def test_greedy_tokens_f32_match_the_reference_engine(gm, qwen_source):
    model = QuantizedTransformer(qwen_source, scheme="int8", dtype=torch.float32)
    assert not model.uses_flash
    got = greedy_generate(model, prompts_of(gm), 32)
    want = gm["qwen_tokens"].tolist()
    identical = 0
    for s in range(len(want)):
        j = first_divergence(got[s], want[s])
        # f32 arithmetic differs from NumPy's only in summation order, so a
        # divergence is allowed only where the reference's top two logits are
        # within 1e-3 of each other (two of the 256 positions)
        assert j is None or gm["qwen_gaps"][s, j] < 1e-3, (s, j, float(gm["qwen_gaps"][s, j]))
        identical += j is None
    assert identical >= 8 - int(np.sum(np.any(gm["qwen_gaps"] < 1e-3, axis=1))), identical


def test_greedy_tokens_f16_teacher_forced_and_free_running(gm, qwen_source):
    model = QuantizedTransformer(qwen_source, scheme="int8", dtype=torch.float16)
    prompts = prompts_of(gm)
    want = gm["qwen_tokens"]
    seqs = [p + want[i].tolist() for i, p in enumerate(prompts)]
    preds, _ = teacher_forced_predictions(model, seqs, [len(p) for p in prompts])
    clear = gm["qwen_gaps"] > TIE_GAP
    pred = np.stack(preds)
    assert np.all(pred[clear] == want[clear]), int(np.sum(pred[clear] != want[clear]))
    got = greedy_generate(model, prompts, 32)
    for s in range(len(prompts)):
        j = first_divergence(got[s], want[s].tolist())
        assert j is None or gm["qwen_gaps"][s, j] <= TIE_GAP, (s, j)
