"""Tensor-parallel communicator: one process per GPU, fused P2P all-reduce.

The reference's "ranks" are list entries in one process and its all_reduce
is a Python sum (ie/parallel/sharding.py:40-44, tensor_parallel.py:68-73).
Here every rank is a process driving its own GPU.  ``ie_comm_create``
allocates this rank's landing buffers and flags; the CUDA IPC handles are
exchanged through ``torch.distributed`` (any backend, host objects only) and
``ie_comm_open`` maps every peer's buffer, after which a row-parallel layer
pushes its partial tiles straight into the peers' memory over NVLink.

Every rank must issue the same collectives in the same order (the epoch that
pairs pushes with waits advances once per call), with the same protocol:
``algo`` is one of ``AR_AUTO`` / ``AR_ONESHOT`` / ``AR_TWOSHOT`` (``ie_tpq.h``
describes both protocols; they give bitwise equal results).  A communicator's
``algo`` attribute is the default of every collective run through it.
"""
from __future__ import annotations

import ctypes

from . import _lib
from .device import dtype_code, require_cuda

AR_AUTO, AR_ONESHOT, AR_TWOSHOT, AR_NVLS = (_lib.IE_AR_AUTO, _lib.IE_AR_ONESHOT,
                                            _lib.IE_AR_TWOSHOT, _lib.IE_AR_NVLS)


def resolve_algo(world_size: int, tiles: int, numel: int, algo: int = AR_AUTO) -> int:
    """The protocol ``algo`` resolves to for a collective of ``world_size``
    ranks over ``tiles`` output tiles and ``numel`` elements (host only)."""
    r = _lib.lib().ie_allreduce_resolve(world_size, tiles, numel, algo)
    if r < 0:
        raise ValueError(f"unknown or unsupported all-reduce algo {algo} (world {world_size})")
    return r


def gather_in_rank_order(own: bytes, world_size: int, group=None) -> bytes:
    """Every rank's ``own`` bytes, concatenated in rank order, through the
    process group (host objects only, so any backend works: gloo on CPU,
    NCCL or gloo beside the GPUs).  All ranks must pass blobs of one length."""
    import torch.distributed as dist

    parts = [None] * world_size
    dist.all_gather_object(parts, own, group=group)
    if any(not isinstance(p, bytes) or len(p) != len(own) for p in parts):
        raise ValueError("every rank must contribute a handle of the same length")
    return b"".join(parts)


class Communicator:
    def __init__(self, rank: int, world_size: int, device=None, max_bytes: int = 64 << 20,
                 group=None, timeout_s: float = 2.0, algo: int = AR_AUTO,
                 _loopback: bool = False):
        torch = require_cuda()
        self.algo = int(algo)
        if world_size < 1:
            raise ValueError("world_size must be at least 1")
        if not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} outside world of {world_size}")
        self.rank = rank
        self.world_size = world_size
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else torch.device(device).index or 0)
        self.max_bytes = int(max_bytes)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().ie_comm_create(rank, world_size, self.device.index, self.max_bytes,
                                             ctypes.byref(h)), "comm_create")
        self._h = h
        mine = ctypes.create_string_buffer(_lib.IE_COMM_HANDLE_BYTES)
        _lib.check(_lib.lib().ie_comm_export(self._h, mine), "comm_export")
        own = mine.raw
        if _loopback or world_size == 1:
            joined = own * world_size
        else:
            joined = gather_in_rank_order(own, world_size, group)
        blob = ctypes.create_string_buffer(joined, world_size * len(own))
        _lib.check(_lib.lib().ie_comm_open(self._h, blob), "comm_open")
        self.set_timeout(timeout_s)
        if not _loopback and world_size > 1:
            import torch.distributed as dist

            dist.barrier(group=group)

    @classmethod
    def loopback(cls, world_size: int = 2, rank: int = 0, **kw) -> "Communicator":
        """A single-GPU communicator whose 'peers' are its own buffer.  No other
        rank ever pushes, so a collective waits for flags nobody sets and ends
        with a timeout status: this is how the bounded-wait path is tested."""
        return cls(rank, world_size, _loopback=True, **kw)

    @property
    def handle(self):
        if self._h is None:
            raise RuntimeError("communicator is closed")
        return self._h

    def set_timeout(self, seconds: float) -> None:
        _lib.check(_lib.lib().ie_comm_set_timeout(self.handle, max(1, int(seconds * 1e9))),
                   "comm_set_timeout")

    def check(self) -> None:
        """Raise ie_tpq._lib.TimeoutError_ if a bounded peer wait ran out."""
        _lib.check(_lib.lib().ie_comm_check(self.handle), "comm")

    def all_reduce(self, tensor, out=None, stream=None, algo: int | None = None):
        """Sum of every rank's ``tensor`` (rank order, f32 arithmetic)."""
        torch = require_cuda()
        t = tensor.contiguous()
        out = torch.empty_like(t) if out is None else out
        _lib.check(_lib.lib().ie_allreduce(self.handle, t.data_ptr(), out.data_ptr(), t.numel(),
                                           dtype_code(t.dtype),
                                           self.algo if algo is None else int(algo),
                                           _lib.stream_ptr(stream)),
                   "allreduce")
        return out

    def close(self) -> None:
        if self._h is not None:
            _lib.lib().ie_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
