"""Quantized checkpoint load path: a HuggingFace safetensors checkpoint
straight into this library's quantized tensor-parallel model.

The reference reads every tensor into host memory as f32, transposes each
projection to ``[in, out]`` and builds its f32 model (ie/load/huggingface.py:
86-139, transpose at :116; reader ie/load/safetensors.py); quantization then
runs over the f32 model.  For a 70B model that is 280 GB of host f32.  Here:

* the safetensors files are memory-mapped (the format: an 8-byte
  little-endian header length, a JSON header of name -> dtype / shape /
  data_offsets, then the raw little-endian data), so a tensor's bytes are read
  from disk only when it is taken, in its stored dtype (bf16 / f16 / f32);
* each projection's bytes go to the GPU as stored and are widened to f32,
  transposed to ``[K, N]`` and quantized there with the reference's tables
  (``quantize_on_device``); the rank's shard is copied out and the full
  weight freed before the next projection;
* the result is a ``QuantizedTransformer`` for one rank.

Names, config fields and the report follow the reference loader
(``layer_names``, ``config_from_hf``, ``LoadReport``), so a checkpoint the
reference loads loads here too.
"""
from __future__ import annotations

import json
import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path
from types import SimpleNamespace

import numpy as np

from .device import require_cuda

HEADER_LEN_BYTES = 8
STORED_DTYPES = {
    "F64": "<f8", "F32": "<f4", "F16": "<f2", "BF16": "<u2", "I64": "<i8", "I32": "<i4",
    "I16": "<i2", "I8": "<i1", "U8": "<u1", "BOOL": "?",
}
SUPPORTED_ARCHITECTURES = {"LlamaForCausalLM", "Qwen2ForCausalLM", "Qwen3ForCausalLM",
                           "MistralForCausalLM", "Gemma2ForCausalLM", "Gemma3ForCausalLM"}
TRANSPOSED = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
OPTIONAL = ("q_bias", "k_bias", "v_bias", "q_norm", "k_norm")


# ---------------------------------------------------------------------------
# safetensors, memory-mapped
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class Entry:
    name: str
    dtype: str
    shape: tuple
    start: int
    end: int

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1


class SafetensorsFile:
    """One ``.safetensors`` file; ``raw(name)`` is a zero-copy view of the
    stored bytes (bf16 as uint16), ``get(name)`` the reference's f32 array."""

    def __init__(self, path) -> None:
        self.path = Path(path)
        if not self.path.exists():
            raise FileNotFoundError(f"no safetensors file at {self.path}")
        with open(self.path, "rb") as fh:
            head = fh.read(HEADER_LEN_BYTES)
            if len(head) != HEADER_LEN_BYTES:
                raise ValueError(f"{self.path} is too short to be a safetensors file")
            (hlen,) = struct.unpack("<Q", head)
            body = fh.read(hlen)
            if len(body) != hlen:
                raise ValueError(f"{self.path}: header of {hlen} bytes is truncated")
            header = json.loads(body)
        self.data_start = HEADER_LEN_BYTES + hlen
        self.entries: dict[str, Entry] = {}
        for name, spec in header.items():
            if name == "__metadata__":
                continue
            s, e = spec["data_offsets"]
            self.entries[name] = Entry(name, spec["dtype"], tuple(spec["shape"]), s, e)
        size = self.path.stat().st_size
        if any(self.data_start + e.end > size for e in self.entries.values()):
            raise ValueError(f"{self.path}: tensor data runs past the end of the file")
        self._map = None

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def __len__(self) -> int:
        return len(self.entries)

    @property
    def names(self) -> list[str]:
        return sorted(self.entries)

    @property
    def total_parameters(self) -> int:
        return sum(e.numel for e in self.entries.values())

    def raw(self, name: str) -> tuple[np.ndarray, str]:
        """(stored-dtype array view over the mapped file, safetensors dtype)."""
        entry = self.entries.get(name)
        if entry is None:
            raise KeyError(f"{name} is not in {self.path.name}")
        if entry.dtype not in STORED_DTYPES:
            raise ValueError(f"unsupported dtype {entry.dtype} for {name}")
        if self._map is None:
            with open(self.path, "rb") as fh:
                self._map = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
        arr = np.frombuffer(self._map, dtype=np.dtype(STORED_DTYPES[entry.dtype]),
                            count=entry.numel, offset=self.data_start + entry.start)
        return arr.reshape(entry.shape), entry.dtype

    def get(self, name: str) -> np.ndarray:
        """The tensor as the reference reads it: f32 (bf16 widened), or its dtype."""
        arr, dt = self.raw(name)
        if dt == "BF16":
            return (arr.astype(np.uint32) << 16).view(np.float32)
        return np.array(arr)


class ShardedCheckpoint:
    """Every ``*.safetensors`` file of a directory as one namespace."""

    def __init__(self, directory) -> None:
        self.directory = Path(directory)
        files = sorted(self.directory.glob("*.safetensors"))
        if not files:
            raise FileNotFoundError(f"no safetensors shards in {self.directory}")
        self.shards = [SafetensorsFile(f) for f in files]
        self.owner = {n: s for s in self.shards for n in s.entries}

    def __contains__(self, name: str) -> bool:
        return name in self.owner

    def __len__(self) -> int:
        return len(self.owner)

    @property
    def names(self) -> list[str]:
        return sorted(self.owner)

    @property
    def total_parameters(self) -> int:
        return sum(s.total_parameters for s in self.shards)

    def _shard(self, name: str) -> SafetensorsFile:
        s = self.owner.get(name)
        if s is None:
            raise KeyError(f"{name} is not in any shard under {self.directory}")
        return s

    def raw(self, name: str):
        return self._shard(name).raw(name)

    def get(self, name: str) -> np.ndarray:
        return self._shard(name).get(name)


def open_checkpoint(directory):
    directory = Path(directory)
    single = directory / "model.safetensors"
    return SafetensorsFile(single) if single.exists() else ShardedCheckpoint(directory)


def write_safetensors(path, tensors: dict) -> None:
    """Write NumPy arrays as a safetensors file (bf16 is not a NumPy dtype:
    pass ``(uint16 array, "BF16")`` for bf16 payloads)."""
    reverse = {np.dtype(v).str: k for k, v in STORED_DTYPES.items() if k != "BF16"}
    header, blobs, off = {}, [], 0
    for name, value in tensors.items():
        arr, dt = value if isinstance(value, tuple) else (value, None)
        arr = np.ascontiguousarray(arr)
        dt = dt or reverse.get(arr.dtype.newbyteorder("<").str)
        if dt is None:
            raise ValueError(f"cannot store dtype {arr.dtype} for {name}")
        payload = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(payload)]}
        blobs.append(payload)
        off += len(payload)
    encoded = json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(encoded)))
        fh.write(encoded)
        for b in blobs:
            fh.write(b)


# ---------------------------------------------------------------------------
# config and names (ie/load/huggingface.py)
# ---------------------------------------------------------------------------
def read_config(directory) -> dict:
    path = Path(directory) / "config.json"
    if not path.exists():
        raise FileNotFoundError(f"no config.json in {directory}")
    return json.loads(path.read_text())


def config_from_hf(raw: dict):
    """ie/load/huggingface.py:31-47 (rotary embedding halved, as HF stores it)."""
    from .model import DecoderConfig

    heads = raw["num_attention_heads"]
    hidden = raw["hidden_size"]
    rope = raw.get("rope_theta") or (raw.get("rope_parameters") or {}).get("rope_theta", 10000.0)
    return DecoderConfig(
        vocab_size=raw["vocab_size"], hidden_size=hidden, num_layers=raw["num_hidden_layers"],
        num_heads=heads, num_kv_heads=raw.get("num_key_value_heads", heads),
        head_dim=raw.get("head_dim", hidden // heads), intermediate_size=raw["intermediate_size"],
        max_position=raw.get("max_position_embeddings", 4096), rope_base=float(rope),
        norm_eps=float(raw.get("rms_norm_eps", 1e-6)), rope_halved=True)


def layer_names(index: int) -> dict[str, str]:
    """ie/load/huggingface.py:50-67."""
    p = f"model.layers.{index}"
    return {
        "attn_norm": f"{p}.input_layernorm.weight", "q_proj": f"{p}.self_attn.q_proj.weight",
        "k_proj": f"{p}.self_attn.k_proj.weight", "v_proj": f"{p}.self_attn.v_proj.weight",
        "o_proj": f"{p}.self_attn.o_proj.weight", "q_bias": f"{p}.self_attn.q_proj.bias",
        "k_bias": f"{p}.self_attn.k_proj.bias", "v_bias": f"{p}.self_attn.v_proj.bias",
        "q_norm": f"{p}.self_attn.q_norm.weight", "k_norm": f"{p}.self_attn.k_norm.weight",
        "mlp_norm": f"{p}.post_attention_layernorm.weight",
        "gate_proj": f"{p}.mlp.gate_proj.weight", "up_proj": f"{p}.mlp.up_proj.weight",
        "down_proj": f"{p}.mlp.down_proj.weight",
    }


@dataclass
class LoadReport:
    """ie/load/huggingface.py:16-27."""
    architecture: str
    parameters: int
    layers_loaded: int
    tied_embeddings: bool
    missing: list = field(default_factory=list)
    unexpected: list = field(default_factory=list)

    @property
    def is_complete(self) -> bool:
        return not self.missing


# ---------------------------------------------------------------------------
# checkpoint -> quantized tensor-parallel model
# ---------------------------------------------------------------------------
def _to_device_f32(ckpt, name: str, device):
    """A stored tensor on the device as f32 (bf16 widened there)."""
    torch = require_cuda()
    arr, dt = ckpt.raw(name)
    t = torch.from_numpy(np.ascontiguousarray(arr)).to(device)
    if dt == "BF16":
        return (t.to(torch.int32) << 16).view(torch.float32)
    return t.to(torch.float32)


def load_quantized(directory, scheme: str = "int8", *, axis: int | None = 0, shard=None,
                   comm=None, device="cuda", dtype=None, quantize_lm_head: bool = False):
    """(QuantizedTransformer for ``shard``, LoadReport) from a HuggingFace
    checkpoint directory.  Each projection is transposed to the reference's
    ``[K, N]`` and quantized on the device with the reference's tables
    (the same codes and scales as ``quantize_transformer`` on the reference's
    loaded f32 model), then sharded as ``QuantizedTransformer`` shards it."""
    torch = require_cuda()
    from .model import QuantizedTransformer, rope_tables_on_device
    from .packed import quantize_on_device

    raw = read_config(directory)
    archs = raw.get("architectures", [])
    config = config_from_hf(raw)
    ckpt = open_checkpoint(directory)
    device = torch.device(device)
    dtype = dtype or torch.bfloat16
    missing, consumed = [], set()

    def take(name, optional=False):
        if name not in ckpt:
            if not optional:
                missing.append(name)
            return None
        consumed.add(name)
        return _to_device_f32(ckpt, name, device)

    def blocks():
        for i in range(config.num_layers):
            names = layer_names(i)
            b = SimpleNamespace(config=config)
            for attr, name in names.items():
                w = take(name, optional=attr in OPTIONAL)
                if w is not None and attr in TRANSPOSED:
                    w = quantize_on_device(w.t().contiguous(), scheme, axis)   # [K, N]
                setattr(b, attr, w)
            for attr in TRANSPOSED + ("attn_norm", "mlp_norm"):
                if getattr(b, attr, None) is None:
                    raise ValueError(f"layer {i}: {names[attr]} is missing from the checkpoint")
            yield b

    embedding = take("model.embed_tokens.weight")
    final_norm = take("model.norm.weight")
    tied = bool(raw.get("tie_word_embeddings", False)) or "lm_head.weight" not in ckpt
    if tied:
        lm_head = embedding.t() if embedding is not None else None
    else:
        head = take("lm_head.weight")
        lm_head = head.t() if head is not None else None
    if embedding is None or final_norm is None or lm_head is None:
        raise ValueError(f"checkpoint lacks {missing}")
    cos, sin = rope_tables_on_device(config.max_position, config.head_dim, config.rope_base,
                                     device)
    source = SimpleNamespace(config=config, blocks=blocks(), embedding=embedding,
                             final_norm=final_norm, lm_head=lm_head, cos=cos, sin=sin)
    model = QuantizedTransformer(source, scheme=scheme, axis=axis, shard=shard, comm=comm,
                                 device=device, dtype=dtype, quantize_lm_head=quantize_lm_head)
    unexpected = sorted(n for n in ckpt.names if n not in consumed and not n.endswith(".inv_freq"))
    report = LoadReport(architecture=archs[0] if archs else "unknown",
                        parameters=ckpt.total_parameters, layers_loaded=config.num_layers,
                        tied_embeddings=tied, missing=missing, unexpected=unexpected)
    return model, report


__all__ = ["SafetensorsFile", "ShardedCheckpoint", "open_checkpoint", "write_safetensors",
           "read_config", "config_from_hf", "layer_names", "LoadReport", "load_quantized"]
