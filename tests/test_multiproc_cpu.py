"""The N > 1 host path on CPU: two processes joined by a gloo process group
(world size 2, 127.0.0.1), as the GPU ranks are joined beside NCCL.

* The communicator's handle exchange returns every rank's handle in rank
  order on every rank (the fused all-reduce maps peers by that order).
* Row-parallel: each process takes its K shard of x and W with the mirror's
  ``Shard`` / ``split_input_dim`` (NumPy weights, and the oracle's int8
  per-K and int4 group-128 tables held in the mirror's ``QuantizedWeight``),
  computes its partial, and the partials gathered across processes and
  summed in rank order equal the oracle's single-process
  ``row_parallel_allreduce`` bit for bit and the unsharded layer within 1e-4
  (the reference's own tolerance, tests/test_tensor_parallel.py:59-72).
* Column-parallel: the N shards gathered across processes reassemble the
  unsharded output exactly (tests/test_tensor_parallel.py:37-56)."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for _p in (REPO, REPO / "inference-engine_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, port: int, world: int) -> None:
    import datetime

    import torch.distributed as dist

    from ie_tpq.comm import gather_in_rank_order
    from ie_tpq.sharding import Shard, split_input_dim, split_output_dim
    from ie_tpq.weights import QuantizedWeight
    from oracle import tpq_oracle as o

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # handle exchange: rank order on every rank
        joined = gather_in_rank_order(bytes([rank + 1]) * 16, world)
        assert joined == b"".join(bytes([r + 1]) * 16 for r in range(world)), joined

        shard = Shard(rank, world)
        m, k, n = 8, 256, 96
        w = o.seeded_weight(k, n, seed=5)
        x = o.seeded_activations(m, k, seed=6)

        # row-parallel, f32 weights
        x_shard = x[:, shard.slice_of(k)]
        partial = x_shard @ split_input_dim(w, shard)
        parts = [None] * world
        dist.all_gather_object(parts, partial)
        total = o.all_reduce(parts)
        assert np.array_equal(total, o.row_parallel_allreduce(x, w, world))
        np.testing.assert_allclose(total, x @ w, rtol=1e-4, atol=1e-4)

        # row-parallel, int8 per-K tables sharded with their rows
        q = o.quantize_integer(w, 8, True, 0)
        qw = QuantizedWeight(codes=q.codes, scale=q.scale, zero_point=None, format_name="int8",
                             bits=8, original_shape=q.codes.shape, group_size=None)
        part_w = split_input_dim(qw, shard)
        q_partial = x_shard @ o.OracleQuantized(part_w.codes, part_w.scale, None, 8).dequantized()
        parts = [None] * world
        dist.all_gather_object(parts, q_partial)
        np.testing.assert_allclose(o.all_reduce(parts), x @ q.dequantized(), rtol=1e-4,
                                   atol=1e-4)

        # row-parallel, int4 group-128 tables: a rank's K shard keeps whole groups
        g = o.quantize_int4_group128(w)
        gw = QuantizedWeight(codes=g.codes, scale=g.scale, zero_point=g.zero, format_name="int4",
                             bits=4, original_shape=(k, n), group_size=128)
        part_g = split_input_dim(gw, shard)
        g_partial = x_shard @ o.OracleGroup128(part_g.codes, part_g.scale,
                                               part_g.zero_point).dequantized()
        parts = [None] * world
        dist.all_gather_object(parts, g_partial)
        np.testing.assert_allclose(o.all_reduce(parts), x @ g.dequantized(), rtol=1e-4,
                                   atol=1e-4)

        # column-parallel: the output shards reassemble the whole output
        col = x @ split_output_dim(w, shard)
        cols = [None] * world
        dist.all_gather_object(cols, col)
        assert np.array_equal(np.concatenate(cols, axis=-1),
                              np.concatenate([x @ w[:, Shard(r, world).slice_of(n)]
                                              for r in range(world)], axis=-1))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce_in_rank_order():
    import torch.multiprocessing as mp

    ctx = mp.start_processes(_rank_main, args=(_free_port(), WORLD), nprocs=WORLD,
                             join=False, start_method="spawn")
    try:
        while not ctx.join(timeout=120):
            pass
    except mp.ProcessRaisedException as e:   # a rank's assertion, with its traceback
        pytest.fail(str(e))
