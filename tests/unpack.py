"""NumPy decoders of the packed device layouts (test-side checkers only)."""
from __future__ import annotations

import numpy as np

PERM = np.array([0, 2, 4, 6, 1, 3, 5, 7])


def unpack_int4(packed: np.ndarray, k: int) -> np.ndarray:
    """[n][k/2] bytes -> [n][k] nibble values (stored codes)."""
    n = packed.shape[0]
    words = packed.reshape(n, -1).view(np.uint32).reshape(n, k // 8)
    out = np.empty((n, k // 8, 8), dtype=np.int32)
    for p in range(8):
        out[:, :, PERM[p]] = (words >> (4 * p)) & 0xF
    return out.reshape(n, k)


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    b = b.astype(np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e - 7))
    return (sign * val).astype(np.float32)


def nearest_e4m3(v: np.ndarray) -> np.ndarray:
    """Round f32 values to the nearest finite e4m3 value (ties to even code)."""
    table = e4m3_to_f32(np.arange(256, dtype=np.uint8))
    finite = np.array([i for i in range(256) if (i & 0x7F) != 0x7F])
    vals = table[finite]
    order = np.argsort(vals, kind="stable")
    vals, codes = vals[order], finite[order]
    flat = v.reshape(-1)
    idx = np.searchsorted(vals, flat)
    idx = np.clip(idx, 1, len(vals) - 1)
    lo, hi = vals[idx - 1], vals[idx]
    pick_hi = (hi - flat) < (flat - lo)
    tie = (hi - flat) == (flat - lo)
    even_hi = (codes[idx] & 1) == 0
    pick_hi = pick_hi | (tie & even_hi)
    out = np.where(pick_hi, hi, lo)
    return out.reshape(v.shape).astype(np.float32)
