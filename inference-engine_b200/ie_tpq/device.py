"""Device plumbing shared by the host modules: moving NumPy inputs into CUDA
memory and checking that a GPU is there.  There is no CPU path: every
function here raises ``RuntimeError`` when CUDA is unavailable."""
from __future__ import annotations

import numpy as np

from . import _lib


def require_cuda():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("the quantized TP path runs on CUDA only and no GPU is visible "
                           "(there is no CPU fallback)")
    _lib.lib()
    return torch


def to_device_f32(x):
    """(contiguous f32 CUDA tensor, input-was-numpy, original shape)."""
    torch = require_cuda()
    if isinstance(x, np.ndarray) or np.isscalar(x):
        arr = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
        return torch.from_numpy(arr).cuda().reshape(-1), True, arr.shape
    if isinstance(x, torch.Tensor):
        shape = tuple(x.shape)
        t = x if x.is_cuda else x.cuda()
        return t.to(torch.float32).contiguous().reshape(-1), False, shape
    raise TypeError(f"expected a NumPy array or a torch tensor, got {type(x).__name__}")


def dtype_code(dtype) -> int:
    import torch

    table = {torch.bfloat16: _lib.IE_DT_BF16, torch.float16: _lib.IE_DT_F16,
             torch.float32: _lib.IE_DT_F32}
    if dtype not in table:
        raise ValueError(f"unsupported dtype {dtype}; expected bfloat16, float16 or float32")
    return table[dtype]
