"""Multi-GPU parity of the fused row-parallel linear + all-reduce: one process
per GPU (spawned here), handles exchanged over a gloo group, partials pushed
over NVLink by the kernel.  Every rank's output must equal the oracle's
rank-order all_reduce of the reference partials and be bitwise identical
across ranks.  Skipped with fewer than two GPUs."""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    from ie_tpq import formats as F
    from ie_tpq import weights as W
    from ie_tpq.comm import Communicator
    from ie_tpq.linear import qlinear
    from ie_tpq.sharding import Shard, split_input_dim
    from oracle import tpq_oracle as o

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    comm = Communicator(rank, world, max_bytes=8 << 20, timeout_s=5.0)
    results = {}
    for scheme, k, n, m in (("int4-g128", 1024, 512, 4), ("int8", 512, 256, 3),
                            ("fp8", 512, 384, 1), ("int8", 256, 128, 17)):
        w = o.seeded_weight(k, n, seed=k + n)
        x = o.seeded_activations(m, k, seed=m)
        res = o.seeded_activations(m, n, seed=m + 7)
        if scheme == "int4-g128":
            q = W.quantize_grouped(w)
        elif scheme == "int8":
            q = W.quantize_integer(w, F.INT8, 0)
        else:
            q = W.quantize_float(w, F.FP8_E4M3, 1)
        sh = Shard(rank, world)
        shard = split_input_dim(q, sh).packed()
        xs = torch.from_numpy(np.ascontiguousarray(x[:, sh.slice_of(k)])).cuda()
        y = None
        for _ in range(3):
            y = qlinear(xs, shard, residual=torch.from_numpy(res).cuda(), comm=comm)
        comm.check()
        results[f"{scheme}_{k}_{n}_{m}"] = y.cpu().numpy()
        # standalone all-reduce of the same partial
        part = qlinear(xs, shard)
        red = comm.all_reduce(part)
        comm.check()
        results[f"ar_{scheme}_{k}_{n}_{m}"] = red.cpu().numpy()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **results)
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


def test_fused_row_parallel_allreduce_across_gpus():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least two GPUs")
    world = min(world, 8)
    import socket

    import torch.multiprocessing as mp

    from oracle import tpq_oracle as o

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, world, port, d)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        outs = [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(world)]
    for key in outs[0]:
        for r in range(1, world):
            assert np.array_equal(outs[0][key], outs[r][key]), key
    for scheme, k, n, m in (("int4-g128", 1024, 512, 4), ("int8", 512, 256, 3),
                            ("fp8", 512, 384, 1), ("int8", 256, 128, 17)):
        w = o.seeded_weight(k, n, seed=k + n)
        x = o.seeded_activations(m, k, seed=m)
        res = o.seeded_activations(m, n, seed=m + 7)
        if scheme == "int4-g128":
            deq = o.quantize_int4_group128(w).dequantized()
        elif scheme == "int8":
            deq = o.quantize_integer(w, 8, True, 0).dequantized()
        else:
            deq = o.quantize_float(w, *o.E4M3, axis=1).dequantized()
        want = res + o.row_parallel_allreduce(x, deq, world)
        np.testing.assert_allclose(outs[0][f"{scheme}_{k}_{n}_{m}"], want, rtol=2e-3, atol=2e-3)
        np.testing.assert_allclose(outs[0][f"ar_{scheme}_{k}_{n}_{m}"], want - res, rtol=2e-3,
                                   atol=2e-3)
