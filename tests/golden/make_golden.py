"""Generate the golden fixtures that pin the CPU oracle to the reference engine.

Run from the repository root, in a container where the reference engine
(kuluruvineeth/inference-engine, pure Python) is importable:

    IE_REFERENCE=/path/to/inference-engine python tests/golden/make_golden.py

It imports the reference's own ``ie.quant`` and ``ie.parallel`` modules, runs
them on seeded inputs and writes

  * ``tests/golden/golden_small.npz`` -- inputs and outputs of the reference at
    sizes small enough to commit (formats, rounding, quantizer tables, shards,
    sharded SwiGLU MLP, row-parallel all-reduce), and
  * ``tests/golden/golden_hashes.json`` -- SHA-256 digests of the reference's
    tables and output for the full-size CPU case (hidden 896, intermediate
    4864, 64 tokens, TP=2, int8 per-channel), whose arrays are too large to
    commit.

The GPU box never runs this script; the tests read only its outputs.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


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

    from ie.parallel import sharding as S
    from ie.parallel.tensor_parallel import ShardedMLP
    from ie.model.transformer import ModelConfig, TransformerBlock
    from ie.quant import formats as F
    from ie.quant import weights as W
    from ie.quant.model import quantize_tensor

    out: dict[str, np.ndarray] = {}

    # --- formats (ie/quant/formats.py) ---------------------------------
    out["fmt_int"] = np.array([F.INT8.signed_max, F.INT8.signed_min, F.INT8.unsigned_max,
                               F.INT4.signed_max, F.INT4.signed_min, F.INT4.unsigned_max],
                              dtype=np.int64)
    out["fmt_float"] = np.array([F.FP8_E4M3.max_value, F.FP8_E4M3.min_normal,
                                 F.FP8_E5M2.max_value, F.FP8_E5M2.min_normal], dtype=np.float64)

    rng = np.random.default_rng(11)
    specials = np.array([0.0, -0.0, 1.0, 1.0625, 1.125, 1.25, 1.375, 2.5, -3.75, 1e6, -1e6,
                         448.0, 449.0, 464.0, 480.0, 2.0 ** -6, 2.0 ** -7, 2.0 ** -8,
                         2.0 ** -9, 2.0 ** -10, 0.00244140625, 0.0029296875, 0.00341796875,
                         5 * 2.0 ** -11, 7 * 2.0 ** -11, 6 * 2.0 ** -11, 5 * 2.0 ** -10,
                         -5 * 2.0 ** -10, 3 * 2.0 ** -10],
                        dtype=np.float32)
    sweep = np.concatenate([specials,
                            (rng.standard_normal(2048) * 40).astype(np.float32),
                            (rng.standard_normal(512) * 0.01).astype(np.float32)])
    out["round_in"] = sweep
    out["round_e4m3"] = F.round_to_float_format(sweep, F.FP8_E4M3).astype(np.float32)
    out["round_e5m2"] = F.round_to_float_format(sweep, F.FP8_E5M2).astype(np.float32)

    # --- weight quantizer tables (ie/quant/weights.py) ------------------
    w = (np.random.default_rng(0).standard_normal((64, 96)) * 0.02).astype(np.float32)
    out["w"] = w
    for tag, axis in (("k", 0), ("n", 1), ("t", None)):
        q = W.quantize_integer(w, F.INT8, axis)
        out[f"int8_{tag}_codes"] = q.codes.astype(np.int8)
        out[f"int8_{tag}_scale"] = q.scale
        out[f"int8_{tag}_deq"] = q.dequantized()
        q = W.quantize_integer(w, F.INT8_ASYM, axis)
        out[f"int8a_{tag}_codes"] = q.codes.astype(np.uint8)
        out[f"int8a_{tag}_scale"] = q.scale
        out[f"int8a_{tag}_zero"] = q.zero_point
        q = W.quantize_integer(w, F.INT4, axis)
        out[f"int4_{tag}_codes"] = q.codes.astype(np.int8)
        out[f"int4_{tag}_scale"] = q.scale
        q = W.quantize_float(w, F.FP8_E4M3, axis)
        out[f"fp8_{tag}_codes"] = q.codes
        out[f"fp8_{tag}_scale"] = q.scale
        out[f"fp8_{tag}_deq"] = q.dequantized()
    q = W.quantize_integer(w, F.INT8)
    out["int8_k_stored_bytes"] = np.array([q.stored_bytes, q.compression])

    # int4 asymmetric group-128 through the reference's own function on a view
    wg = (np.random.default_rng(1).standard_normal((256, 192)) * 0.02).astype(np.float32)
    out["wg"] = wg
    view = np.ascontiguousarray(wg.T).reshape(-1, 128)
    q = W.quantize_integer(view, F.IntegerFormat(4, symmetric=False), 0)
    out["g128_codes"] = q.codes.astype(np.uint8)
    out["g128_scale"] = q.scale
    out["g128_zero"] = q.zero_point
    out["g128_deq"] = q.dequantized()

    # per-token fp8 activations through quantize_float(x, FP8_E4M3, axis=0)
    xa = np.random.default_rng(2).standard_normal((6, 256)).astype(np.float32)
    out["act_x"] = xa
    q = W.quantize_float(xa, F.FP8_E4M3, 0)
    out["act_codes"] = q.codes
    out["act_scale"] = q.scale

    # edge weights (tests/test_quantization.py:111-119 and the outlier column)
    const = np.full((4, 4), 0.25, dtype=np.float32)
    zeros = np.zeros((4, 4), dtype=np.float32)
    onesided = (np.abs(np.random.default_rng(3).standard_normal((8, 16))) + 1.0).astype(np.float32)
    outlier = np.random.default_rng(4).standard_normal((16, 32)).astype(np.float32)
    outlier[:, 0] *= 500.0
    for name, arr in (("const", const), ("zeros", zeros), ("onesided", onesided),
                      ("outlier", outlier)):
        out[f"edge_{name}"] = arr
        q = W.quantize_integer(arr, F.INT8)
        out[f"edge_{name}_int8_codes"] = q.codes.astype(np.int8)
        out[f"edge_{name}_int8_scale"] = q.scale
        q = W.quantize_integer(arr, F.INT8_ASYM, None)
        out[f"edge_{name}_int8a_codes"] = q.codes.astype(np.uint8)
        out[f"edge_{name}_int8a_scale"] = q.scale
        out[f"edge_{name}_int8a_zero"] = q.zero_point
        q = W.quantize_float(arr, F.FP8_E4M3)
        out[f"edge_{name}_fp8_codes"] = q.codes
        out[f"edge_{name}_fp8_scale"] = q.scale

    # --- sharding (ie/parallel/sharding.py) -----------------------------
    base = np.arange(12 * 24, dtype=np.float32).reshape(12, 24)
    out["shard_base"] = base
    for world in (1, 2, 3, 4):
        for r in range(world):
            out[f"col_{world}_{r}"] = np.ascontiguousarray(S.split_output_dim(base, S.Shard(r, world)))
            out[f"row_{world}_{r}"] = np.ascontiguousarray(S.split_input_dim(base, S.Shard(r, world)))
    for world in (1, 2, 4):
        for r in range(world):
            out[f"heads_{world}_{r}"] = np.ascontiguousarray(
                S.split_heads(base, S.Shard(r, world), 4, 6))

    # --- sharded SwiGLU MLP (ie/parallel/tensor_parallel.py:46-56) -------
    cfg = ModelConfig(vocab_size=64, hidden_size=64, num_layers=1, num_heads=4,
                      num_kv_heads=2, head_dim=16, intermediate_size=256)
    block = TransformerBlock(cfg, np.random.default_rng(5))
    for name in ("gate_proj", "up_proj", "down_proj"):
        setattr(block, name, quantize_tensor(getattr(block, name), F.INT8).dequantized())
    xm = np.random.default_rng(6).standard_normal((8, 64)).astype(np.float32)
    out["mlp_x"] = xm
    out["mlp_gate"], out["mlp_up"], out["mlp_down"] = block.gate_proj, block.up_proj, block.down_proj
    for world in (1, 2, 4):
        partials = [ShardedMLP(block, S.Shard(r, world)).forward(xm) for r in range(world)]
        out[f"mlp_out_{world}"] = xm + S.all_reduce(partials)

    # --- row-parallel linear + all_reduce on int4-g128 dequantized weights ---
    wr = (np.random.default_rng(7).standard_normal((512, 64)) * 0.02).astype(np.float32)
    view = np.ascontiguousarray(wr.T).reshape(-1, 128)
    q = W.quantize_integer(view, F.IntegerFormat(4, symmetric=False), 0)
    wr_deq = q.dequantized().reshape(64, 512).T.copy()
    xr = np.random.default_rng(8).standard_normal((5, 512)).astype(np.float32)
    out["row_w"], out["row_x"] = wr, xr
    for world in (1, 2, 4):
        partials = []
        for r in range(world):
            sh = S.Shard(r, world)
            partials.append(S.RowParallelLinear(wr_deq, sh).forward(xr[:, sh.slice_of(512)]))
        out[f"row_out_{world}"] = S.all_reduce(partials)

    np.savez_compressed(HERE / "golden_small.npz", **out)

    # --- the full-size CPU case: digests only ----------------------------
    rng = np.random.default_rng(0)
    hidden, inter, tokens = 896, 4864, 64
    gate = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)
    up = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)
    down = (rng.standard_normal((inter, hidden)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, hidden)).astype(np.float32)
    hashes = {}
    block = TransformerBlock(ModelConfig(vocab_size=64, hidden_size=hidden, num_layers=1,
                                         num_heads=14, num_kv_heads=2, head_dim=64,
                                         intermediate_size=inter), np.random.default_rng(0))
    for name, wt in (("gate", gate), ("up", up), ("down", down)):
        q = quantize_tensor(wt, F.INT8)
        hashes[f"config1_{name}_codes"] = digest(q.codes)
        hashes[f"config1_{name}_scale"] = digest(q.scale)
        setattr(block, f"{name}_proj", q.dequantized())
    partials = [ShardedMLP(block, S.Shard(r, 2)).forward(x) for r in range(2)]
    y = x + S.all_reduce(partials)
    hashes["config1_out_tp2"] = digest(y)
    hashes["config1_out_tp2_sum"] = float(np.sum(y.astype(np.float64)))
    hashes["config1_out_tp2_absmax"] = float(np.max(np.abs(y)))
    q = W.quantize_integer(np.ascontiguousarray(down.T).reshape(-1, 128),
                           F.IntegerFormat(4, symmetric=False), 0)
    hashes["config1_down_g128_codes"] = digest(q.codes)
    hashes["config1_down_g128_scale"] = digest(q.scale)
    hashes["config1_down_g128_zero"] = digest(q.zero_point)
    q = W.quantize_float(down, F.FP8_E4M3)
    hashes["config1_down_fp8_codes"] = digest(q.codes)
    hashes["config1_down_fp8_scale"] = digest(q.scale)
    (HERE / "golden_hashes.json").write_text(json.dumps(hashes, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(out)} arrays and {len(hashes)} digests")


if __name__ == "__main__":
    main()
