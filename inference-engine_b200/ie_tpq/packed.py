"""Packed device weights: the HBM layout the kernels stream.

A reference weight is ``[K, N]`` with ``y = x @ W`` (ie/model/transformer.py:48-61).
On the device every output column becomes a K-contiguous row:

  * int8   -- ``codes[n][k]`` int8 (reference codes, [-127, 127]);
  * fp8    -- ``codes[n][k]`` e4m3 bytes of the reference's f32 codes;
  * int4   -- ``codes[n][k/2]``; each 32-bit word covers 8 consecutive k with
              nibble p holding k0 + (0,2,4,6,1,3,5,7)[p] so one mask+or yields
              the (k0+2p, k0+2p+1) pair; symmetric codes are stored +8;
  * scales -- f32 ``[K]`` (reference axis 0), ``[N]`` (axis 1) or ``[1]``;
              group-128: f16 scale and zero ``[K/128][N]`` (a documented cast of
              the reference's bit-exact f32 tables, N-contiguous per K group).

Gate/up pairs for the fused SiLU*up epilogue interleave rows (row 2j = gate
column j, row 2j+1 = up column j); per-K and per-tensor tables then hold the
gate table followed by the up table.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from .device import require_cuda

_FMT_NAMES = {_lib.IE_FMT_INT8: "int8", _lib.IE_FMT_INT4: "int4", _lib.IE_FMT_FP8_E4M3: "fp8-e4m3"}
_AXIS_NAMES = {_lib.IE_AXIS_K: "k", _lib.IE_AXIS_N: "n", _lib.IE_AXIS_TENSOR: "tensor",
               _lib.IE_AXIS_GROUP128: "group128"}


def _adjacent(scale, zero) -> bool:
    return (scale.is_contiguous() and zero.is_contiguous() and scale.shape == zero.shape
            and zero.data_ptr() == scale.data_ptr() + scale.numel() * scale.element_size())


def torch_empty_like_pair(t):
    torch = require_cuda()
    return torch.empty((2,) + tuple(t.shape), dtype=t.dtype, device=t.device)


class PackedWeight:
    """A quantized ``[K, N]`` weight resident in device memory."""

    def __init__(self, *, fmt: int, axis: int, k: int, n: int, codes, scale, zero=None,
                 int4_symmetric: bool = False, gate_up: bool = False, unrepresentable: int = 0,
                 act_quant: int = 0):
        self.fmt = fmt
        self.axis = axis
        self.k = int(k)
        self.n = int(n)
        self.codes = codes
        if zero is not None and scale.dim() == 2 and not _adjacent(scale, zero):
            # group tables live in one [2][G][N] array (scale, then zero) so the
            # tensor-core kernel fetches both with a single copy per stage
            joint = torch_empty_like_pair(scale)
            joint[0].copy_(scale)
            joint[1].copy_(zero)
            scale, zero = joint[0], joint[1]
        self.scale = scale
        self.zero = zero
        self.int4_symmetric = bool(int4_symmetric)
        self.gate_up = bool(gate_up)
        self.unrepresentable = int(unrepresentable)
        # how activations meet this weight (ie_qlinear_args.act_quant): 0 as
        # given, IE_ACT_FP8_TOKEN per-token e4m3 (the "fp8-native" scheme)
        self.act_quant = int(act_quant)
        self._struct = None

    # ---- description -----------------------------------------------------
    def __repr__(self) -> str:
        return (f"PackedWeight({_FMT_NAMES[self.fmt]}, axis={_AXIS_NAMES[self.axis]}, "
                f"K={self.k}, N={self.n}{', gate_up' if self.gate_up else ''})")

    @property
    def device(self):
        return self.codes.device

    @property
    def out_features(self) -> int:
        return self.n // 2 if self.gate_up else self.n

    @property
    def nbytes(self) -> int:
        """Bytes of HBM the weight occupies (codes + tables)."""
        total = self.codes.numel() * self.codes.element_size()
        total += self.scale.numel() * self.scale.element_size()
        if self.zero is not None:
            total += self.zero.numel() * self.zero.element_size()
        return int(total)

    def qweight(self) -> _lib.QWeight:
        if self._struct is None:
            self._struct = _lib.QWeight(
                format=self.fmt, axis=self.axis, k=self.k, n=self.n,
                codes=self.codes.data_ptr(), scale=self.scale.data_ptr(),
                zero=self.zero.data_ptr() if self.zero is not None else None,
                int4_symmetric=int(self.int4_symmetric), gate_up=int(self.gate_up))
        return self._struct

    # ---- construction ------------------------------------------------------
    @classmethod
    def from_quantized(cls, qw, device=None) -> "PackedWeight":
        """Pack a reference-format ``QuantizedWeight`` (host tables) on the device."""
        torch = require_cuda()
        dev = torch.device(device) if device is not None else torch.device("cuda",
                                                                            torch.cuda.current_device())
        if qw.group_size:
            n, k = qw.codes.shape
            fmt, axis, sym = _lib.IE_FMT_INT4, _lib.IE_AXIS_GROUP128, False
        else:
            if qw.codes.ndim != 2:
                raise ValueError("only 2-D [K, N] weights have a packed device layout")
            k, n = qw.codes.shape
            if qw.codes.dtype == np.float32:
                if qw.bits != 8:
                    raise ValueError(f"{qw.format_name} has no packed device layout (fp8-e4m3 only)")
                if not qw.format_name.startswith("fp8-e4m3"):
                    raise ValueError(f"{qw.format_name} has no packed device layout (fp8-e4m3 only)")
                fmt = _lib.IE_FMT_FP8_E4M3
            elif qw.bits == 8:
                fmt = _lib.IE_FMT_INT8
            elif qw.bits == 4:
                fmt = _lib.IE_FMT_INT4
            else:
                raise ValueError(f"{qw.format_name} has no packed device layout")
            if qw.zero_point is not None:
                raise ValueError(f"{qw.format_name}: asymmetric per-axis codes have no packed "
                                 "layout (use int8 symmetric, int4 group-128 or fp8)")
            sym = fmt == _lib.IE_FMT_INT4
            shape = tuple(qw.scale.shape)
            if qw.scale.size == 1:
                axis = _lib.IE_AXIS_TENSOR
            elif shape == (k, 1):
                axis = _lib.IE_AXIS_K
            elif shape == (1, n):
                axis = _lib.IE_AXIS_N
            else:
                raise ValueError(f"scale of shape {shape} does not match a [{k}, {n}] weight")
        torch.cuda.set_device(dev)
        stream = _lib.stream_ptr()
        codes_src = torch.from_numpy(np.ascontiguousarray(qw.codes)).to(dev)
        counter = torch.zeros(1, dtype=torch.int32, device=dev)
        row_bytes = k // 2 if fmt == _lib.IE_FMT_INT4 else k
        codes = torch.empty((n, row_bytes), dtype=torch.uint8, device=dev)
        scale32 = torch.from_numpy(np.ascontiguousarray(qw.scale, dtype=np.float32).reshape(-1)).to(dev)
        zero = None
        if axis == _lib.IE_AXIS_GROUP128:
            zero32 = torch.from_numpy(np.ascontiguousarray(qw.zero_point, dtype=np.float32)
                                      .reshape(-1)).to(dev)
            scale = torch.empty((k // 128, n), dtype=torch.float16, device=dev)
            zero = torch.empty((k // 128, n), dtype=torch.float16, device=dev)
            _lib.check(_lib.lib().ie_pack_weight(
                fmt, axis, 0, k, n, codes_src.data_ptr(), scale32.data_ptr(), zero32.data_ptr(),
                codes.data_ptr(), scale.data_ptr(), zero.data_ptr(), counter.data_ptr(), stream),
                "pack_weight")
        else:
            scale = scale32.clone()
            _lib.check(_lib.lib().ie_pack_weight(
                fmt, axis, int(sym), k, n, codes_src.data_ptr(), None, None, codes.data_ptr(),
                None, None, counter.data_ptr() if fmt == _lib.IE_FMT_FP8_E4M3 else None, stream),
                "pack_weight")
        bad = int(counter.item())
        if axis == _lib.IE_AXIS_GROUP128 and bad:
            raise ValueError(f"{bad} group scale/zero values are not representable in f16")
        return cls(fmt=fmt, axis=axis, k=k, n=n, codes=codes, scale=scale, zero=zero,
                   int4_symmetric=sym, unrepresentable=bad)

    # ---- views ------------------------------------------------------------
    def dequantize(self, layout: str = "kn", dtype=None):
        """Dense weight on the device: ``"kn"`` f32 ``[K, N]`` (the reference's
        ``dequantized()``), or ``"nk"`` ``[N, K]`` of ``dtype`` (for cuBLAS)."""
        torch = require_cuda()
        from .device import dtype_code

        dtype = dtype or torch.float32
        if layout == "kn":
            out = torch.empty((self.k, self.n), dtype=dtype, device=self.device)
            lay = 0
        elif layout == "nk":
            out = torch.empty((self.n, self.k), dtype=dtype, device=self.device)
            lay = 1
        else:
            raise ValueError("layout must be 'kn' or 'nk'")
        q = self.qweight()
        _lib.check(_lib.lib().ie_dequantize(q, lay, dtype_code(dtype), out.data_ptr(),
                                            _lib.stream_ptr()), "dequantize")
        return out

    def slice_rows(self, n0: int, n1: int) -> "PackedWeight":
        """Output columns [n0, n1) of the reference weight (a column shard)."""
        if self.gate_up:
            raise ValueError("shard gate and up before pairing them")
        scale, zero = self.scale, self.zero
        if self.axis == _lib.IE_AXIS_N:
            scale = self.scale[n0:n1]
        elif self.axis == _lib.IE_AXIS_GROUP128:
            scale = self.scale[:, n0:n1].contiguous()
            zero = self.zero[:, n0:n1].contiguous()
        return PackedWeight(fmt=self.fmt, axis=self.axis, k=self.k, n=n1 - n0,
                            codes=self.codes[n0:n1], scale=scale, zero=zero,
                            int4_symmetric=self.int4_symmetric, act_quant=self.act_quant)

    def slice_k(self, k0: int, k1: int) -> "PackedWeight":
        """Input rows [k0, k1) of the reference weight (a row shard); copies."""
        if self.gate_up:
            raise ValueError("shard gate and up before pairing them")
        align = 128 if self.axis == _lib.IE_AXIS_GROUP128 else (
            32 if self.fmt == _lib.IE_FMT_INT4 else 16)
        if k0 % align or k1 % align:
            raise ValueError(f"a K shard of this format must start and end on multiples of {align}")
        per = 2 if self.fmt == _lib.IE_FMT_INT4 else 1
        codes = self.codes[:, k0 // per:k1 // per].contiguous()
        scale, zero = self.scale, self.zero
        if self.axis == _lib.IE_AXIS_K:
            scale = self.scale[k0:k1].contiguous()
        elif self.axis == _lib.IE_AXIS_GROUP128:
            scale = self.scale[k0 // 128:k1 // 128].contiguous()
            zero = self.zero[k0 // 128:k1 // 128].contiguous()
        return PackedWeight(fmt=self.fmt, axis=self.axis, k=k1 - k0, n=self.n, codes=codes,
                            scale=scale, zero=zero, int4_symmetric=self.int4_symmetric,
                            act_quant=self.act_quant)

    @staticmethod
    def pair_gate_up(gate: "PackedWeight", up: "PackedWeight") -> "PackedWeight":
        """Interleave gate and up rows for the fused SiLU*up epilogue."""
        torch = require_cuda()
        if (gate.fmt, gate.axis, gate.k, gate.n, gate.int4_symmetric) != \
                (up.fmt, up.axis, up.k, up.n, up.int4_symmetric):
            raise ValueError("gate and up must share format, scale axis and shape")
        codes = torch.stack([gate.codes, up.codes], dim=1).reshape(2 * gate.n, -1).contiguous()
        zero = None
        if gate.axis in (_lib.IE_AXIS_K, _lib.IE_AXIS_TENSOR):
            scale = torch.cat([gate.scale.reshape(-1), up.scale.reshape(-1)]).contiguous()
        elif gate.axis == _lib.IE_AXIS_N:
            scale = torch.stack([gate.scale, up.scale], dim=1).reshape(2 * gate.n).contiguous()
        else:   # group tables [G][N]: interleave along N
            g = gate.scale.shape[0]
            scale = torch.stack([gate.scale, up.scale], dim=2).reshape(g, 2 * gate.n).contiguous()
            zero = torch.stack([gate.zero, up.zero], dim=2).reshape(g, 2 * gate.n).contiguous()
        return PackedWeight(fmt=gate.fmt, axis=gate.axis, k=gate.k, n=2 * gate.n, codes=codes,
                            scale=scale, zero=zero, int4_symmetric=gate.int4_symmetric,
                            gate_up=True, act_quant=gate.act_quant)


def concat_rows(parts: list["PackedWeight"]) -> "PackedWeight":
    """Stack column shards (e.g. q, k and v heads) into one packed weight.
    Only for tables that live on N (per-N scales, group-128): per-K scales
    differ between the parts and cannot share one row."""
    torch = require_cuda()
    first = parts[0]
    for p in parts:
        if (p.fmt, p.axis, p.k, p.int4_symmetric, p.gate_up) != \
                (first.fmt, first.axis, first.k, first.int4_symmetric, False):
            raise ValueError("concatenated weights must share format, scale axis and K")
    if first.axis not in (_lib.IE_AXIS_N, _lib.IE_AXIS_GROUP128):
        raise ValueError("only per-N or group-128 tables can be concatenated along N")
    dim = 1 if first.axis == _lib.IE_AXIS_GROUP128 else 0
    zero = torch.cat([p.zero for p in parts], dim=1).contiguous() if first.zero is not None else None
    return PackedWeight(fmt=first.fmt, axis=first.axis, k=first.k, n=sum(p.n for p in parts),
                        codes=torch.cat([p.codes for p in parts]).contiguous(),
                        scale=torch.cat([p.scale for p in parts], dim=dim).contiguous(), zero=zero,
                        int4_symmetric=first.int4_symmetric, act_quant=first.act_quant)


def quantize_on_device(w, scheme: str, axis: int | None = 0) -> "PackedWeight":
    """Quantize a ``[K, N]`` f32 CUDA tensor straight into the packed layout.

    ``scheme``: "int8" (symmetric, reference axis), "int4" (symmetric), "fp8"
    (e4m3), "int4-g128", or "fp8-native": e4m3 with one scale per output
    channel (N) whose callers quantize activations per token to e4m3 and
    contract both on the tensor cores (``act_quant``; ``axis`` is ignored).
    The tables are the same as the host path's (``ie_tpq.weights``) but never
    leave the device -- the load path for model-sized weights.
    """
    torch = require_cuda()
    if w.dim() != 2 or w.dtype != torch.float32 or not w.is_cuda:
        raise ValueError("quantize_on_device takes a 2-D float32 CUDA tensor [K, N]")
    k, n = w.shape
    stream = _lib.stream_ptr()
    dev = w.device
    L = _lib.lib()
    if scheme == "int4-g128":
        if k % 128:
            raise ValueError(f"K={k} is not a multiple of 128")
        view = w.t().contiguous().reshape(n * k // 128, 128)
        codes = torch.empty_like(view, dtype=torch.int32)
        s32 = torch.empty(view.shape[0], dtype=torch.float32, device=dev)
        z32 = torch.empty_like(s32)
        _lib.check(L.ie_quantize_integer(view.data_ptr(), view.shape[0], 128, 4, 0, 0,
                                         codes.data_ptr(), s32.data_ptr(), z32.data_ptr(), stream),
                   "quantize_integer")
        del view
        packed = torch.empty((n, k // 2), dtype=torch.uint8, device=dev)
        s16 = torch.empty((k // 128, n), dtype=torch.float16, device=dev)
        z16 = torch.empty_like(s16)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.check(L.ie_pack_weight(_lib.IE_FMT_INT4, _lib.IE_AXIS_GROUP128, 0, k, n,
                                    codes.data_ptr(), s32.data_ptr(), z32.data_ptr(),
                                    packed.data_ptr(), s16.data_ptr(), z16.data_ptr(),
                                    bad.data_ptr(), stream), "pack_weight")
        if int(bad.item()):
            raise ValueError(f"{int(bad.item())} group scale/zero values are not representable in f16")
        return PackedWeight(fmt=_lib.IE_FMT_INT4, axis=_lib.IE_AXIS_GROUP128, k=k, n=n,
                            codes=packed, scale=s16, zero=z16)
    act_quant = 0
    if scheme == "fp8-native":
        scheme, axis, act_quant = "fp8", 1, _lib.IE_ACT_FP8_TOKEN
    kaxis = -1 if axis is None else axis
    nscale = k if kaxis == 0 else (n if kaxis == 1 else 1)
    scale = torch.empty(nscale, dtype=torch.float32, device=dev)
    if scheme == "fp8":
        codes = torch.empty((k, n), dtype=torch.float32, device=dev)
        _lib.check(L.ie_quantize_float(w.data_ptr(), k, n, 4, 3, 0, kaxis, codes.data_ptr(),
                                       scale.data_ptr(), stream), "quantize_float")
        fmt, sym = _lib.IE_FMT_FP8_E4M3, False
    elif scheme in ("int8", "int4"):
        bits = 8 if scheme == "int8" else 4
        codes = torch.empty((k, n), dtype=torch.int32, device=dev)
        _lib.check(L.ie_quantize_integer(w.data_ptr(), k, n, bits, 1, kaxis, codes.data_ptr(),
                                         scale.data_ptr(), None, stream), "quantize_integer")
        fmt, sym = (_lib.IE_FMT_INT8, False) if bits == 8 else (_lib.IE_FMT_INT4, True)
    else:
        raise ValueError(f"unknown scheme {scheme!r}")
    row_bytes = k // 2 if fmt == _lib.IE_FMT_INT4 else k
    packed = torch.empty((n, row_bytes), dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(L.ie_pack_weight(fmt, {0: _lib.IE_AXIS_K, 1: _lib.IE_AXIS_N, -1: _lib.IE_AXIS_TENSOR}[kaxis],
                                int(sym), k, n, codes.data_ptr(), None, None, packed.data_ptr(),
                                None, None, bad.data_ptr() if fmt == _lib.IE_FMT_FP8_E4M3 else None,
                                stream), "pack_weight")
    axis_id = {0: _lib.IE_AXIS_K, 1: _lib.IE_AXIS_N, -1: _lib.IE_AXIS_TENSOR}[kaxis]
    return PackedWeight(fmt=fmt, axis=axis_id, k=k, n=n, codes=packed, scale=scale,
                        int4_symmetric=sym, unrepresentable=int(bad.item()), act_quant=act_quant)
