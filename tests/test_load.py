"""The quantized checkpoint load path (ie_tpq.load) -- the reference's
ie/load/safetensors.py and ie/load/huggingface.py:86-139 restated around a
memory-mapped reader and on-device quantization.

CPU: the safetensors reader against the arrays written (f32, f16, bf16),
sharded checkpoints, the reference's config mapping and error behaviour
(tests/test_loading.py of the reference).  GPU (marked): a synthetic
HuggingFace checkpoint loads into a QuantizedTransformer whose packed shards
hold exactly the oracle's quantization of the transposed weights, and whose
greedy tokens equal the model built from the same weights in memory."""
from __future__ import annotations

import json

import numpy as np
import pytest

from ie_tpq.load import (SafetensorsFile, ShardedCheckpoint, config_from_hf, layer_names,
                         open_checkpoint, read_config, write_safetensors)

HF_CONFIG = {
    "architectures": ["LlamaForCausalLM"],
    "vocab_size": 96, "hidden_size": 256, "num_hidden_layers": 2,
    "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
    "intermediate_size": 512, "max_position_embeddings": 512,
    "rope_theta": 500000.0, "rms_norm_eps": 1e-5, "tie_word_embeddings": False,
}


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns, round to nearest even."""
    u = a.astype(np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def synthetic_checkpoint(directory, raw=None, shards=1, dtype="BF16"):
    raw = dict(raw or HF_CONFIG)
    (directory / "config.json").write_text(json.dumps(raw))
    spec = config_from_hf(raw)
    rng = np.random.default_rng(0)
    normal = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)
    t = {"model.embed_tokens.weight": normal(spec.vocab_size, spec.hidden_size),
         "model.norm.weight": np.ones(spec.hidden_size, np.float32)}
    if not raw.get("tie_word_embeddings"):
        t["lm_head.weight"] = normal(spec.vocab_size, spec.hidden_size)
    q_out, kv_out = spec.num_heads * spec.head_dim, spec.num_kv_heads * spec.head_dim
    for i in range(spec.num_layers):
        n = layer_names(i)
        t[n["attn_norm"]] = np.ones(spec.hidden_size, np.float32)
        t[n["mlp_norm"]] = np.ones(spec.hidden_size, np.float32)
        t[n["q_proj"]] = normal(q_out, spec.hidden_size)
        t[n["k_proj"]] = normal(kv_out, spec.hidden_size)
        t[n["v_proj"]] = normal(kv_out, spec.hidden_size)
        t[n["o_proj"]] = normal(spec.hidden_size, q_out)
        t[n["gate_proj"]] = normal(spec.intermediate_size, spec.hidden_size)
        t[n["up_proj"]] = normal(spec.intermediate_size, spec.hidden_size)
        t[n["down_proj"]] = normal(spec.hidden_size, spec.intermediate_size)
    if dtype == "BF16":   # what the checkpoint stores, and its f32 value
        stored = {k: (bf16_bits(v), "BF16") for k, v in t.items()}
        values = {k: (bf16_bits(v).astype(np.uint32) << 16).view(np.float32) for k, v in t.items()}
    else:
        stored, values = t, t
    names = list(stored)
    per = -(-len(names) // shards)
    for s in range(shards):
        chunk = {k: stored[k] for k in names[s * per:(s + 1) * per]}
        path = directory / ("model.safetensors" if shards == 1
                            else f"model-{s:05d}-of-{shards:05d}.safetensors")
        write_safetensors(path, chunk)
    return values


def test_roundtrip_f32_f16_bf16(tmp_path):
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    h = np.linspace(-2, 2, 7).astype(np.float16)
    b = np.array([1.5, -0.3125, 3.0e5], dtype=np.float32)
    path = tmp_path / "m.safetensors"
    write_safetensors(path, {"a": a, "h": h, "b": (bf16_bits(b), "BF16")})
    f = SafetensorsFile(path)
    assert f.names == ["a", "b", "h"] and len(f) == 3 and f.total_parameters == 16
    assert np.array_equal(f.get("a"), a) and f.get("a").shape == (2, 3)
    assert np.array_equal(f.get("h"), h)
    assert np.array_equal(f.get("b"), (bf16_bits(b).astype(np.uint32) << 16).view(np.float32))
    raw, dt = f.raw("b")
    assert dt == "BF16" and raw.dtype == np.uint16


def test_errors_follow_the_reference(tmp_path):
    path = tmp_path / "m.safetensors"
    write_safetensors(path, {"a": np.zeros(3, np.float32)})
    with pytest.raises(KeyError):
        SafetensorsFile(path).get("nope")
    with pytest.raises(FileNotFoundError):
        SafetensorsFile(tmp_path / "absent.safetensors")
    bad = tmp_path / "short.safetensors"
    bad.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        SafetensorsFile(bad)
    with pytest.raises(FileNotFoundError):
        ShardedCheckpoint(tmp_path / "empty_dir_that_does_not_exist")
    with pytest.raises(FileNotFoundError):
        read_config(tmp_path)


def test_sharded_checkpoint_is_one_namespace(tmp_path):
    values = synthetic_checkpoint(tmp_path, shards=3, dtype="F32")
    ckpt = open_checkpoint(tmp_path)
    assert isinstance(ckpt, ShardedCheckpoint) and len(ckpt.shards) == 3
    assert ckpt.names == sorted(values)
    for name, v in values.items():
        assert np.array_equal(ckpt.get(name), v)


def test_hf_config_mapping():
    spec = config_from_hf(HF_CONFIG)
    assert (spec.num_kv_heads, spec.head_dim, spec.rope_base, spec.norm_eps) == (2, 64, 500000.0,
                                                                                 1e-5)
    assert spec.rope_halved
    raw = dict(HF_CONFIG)
    del raw["head_dim"], raw["rope_theta"]
    raw["rope_parameters"] = {"rope_theta": 1.0e6}
    spec = config_from_hf(raw)
    assert spec.head_dim == 256 // 4 and spec.rope_base == 1.0e6


@pytest.mark.gpu
@pytest.mark.parametrize("scheme", ["int8", "int4-g128"])
def test_loaded_model_matches_the_oracle_and_the_in_memory_model(tmp_path, scheme):
    import torch
    from types import SimpleNamespace

    from ie_tpq.decode import greedy_generate
    from ie_tpq.load import load_quantized
    from ie_tpq.model import QuantizedTransformer, rope_tables_on_device
    from oracle import tpq_oracle as o

    values = synthetic_checkpoint(tmp_path)
    model, report = load_quantized(tmp_path, scheme, dtype=torch.float32)
    assert report.is_complete and report.unexpected == [] and report.layers_loaded == 2
    assert not report.tied_embeddings and report.architecture == "LlamaForCausalLM"
    # the packed o projection of layer 1 is the oracle's quantization of W.T
    w = values[layer_names(1)["o_proj"]].T.copy()
    deq = model.attn[1].o_proj.dequantize().cpu().numpy()
    if scheme == "int8":
        np.testing.assert_array_equal(deq, o.quantize_integer(w, 8, True, 0).dequantized())
    else:   # group tables held as f16
        np.testing.assert_allclose(deq, o.quantize_int4_group128(w).dequantized(), rtol=1e-3,
                                   atol=1e-7)
    # the same weights through the in-memory constructor give the same tokens
    spec = config_from_hf(HF_CONFIG)
    cos, sin = rope_tables_on_device(spec.max_position, spec.head_dim, spec.rope_base, "cuda")
    blocks = []
    for i in range(spec.num_layers):
        n = layer_names(i)
        b = SimpleNamespace(config=spec, q_bias=None, k_bias=None, v_bias=None, q_norm=None,
                            k_norm=None, attn_norm=values[n["attn_norm"]],
                            mlp_norm=values[n["mlp_norm"]])
        for attr in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            setattr(b, attr, values[n[attr]].T.copy())
        blocks.append(b)
    src = SimpleNamespace(config=spec, blocks=blocks, embedding=values["model.embed_tokens.weight"],
                          final_norm=values["model.norm.weight"],
                          lm_head=values["lm_head.weight"].T.copy(), cos=cos, sin=sin)
    mem = QuantizedTransformer(src, scheme=scheme, dtype=torch.float32)
    prompts = [[1, 5, 9, 2], [7, 3]]
    assert greedy_generate(model, prompts, 6) == greedy_generate(mem, prompts, 6)
