"""Benchmark of the tensor-parallel quantized linear path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one process per GPU)

Workload (the headline config: the int4 Llama-3-8B-shaped decoder): one
decode step of the whole model's quantized linear path -- 32 layers x
{rms_norm + qkv (column; the norm folded into the GEMM), o (row + fused
all-reduce + residual), rms_norm + gate/up (column, folded norm, fused
SiLU*up), down (row + fused all-reduce + residual)} --
for a decode batch of 16 tokens, int4 asymmetric group-128 weights (f16
scales/zeros), bf16 activations, tensor-parallel over N GPUs (TP=N, total work
fixed: strong scaling).  Attention is outside the path (see ie_tpq.stack).

``value`` = tokens/s of the step with inputs resident in HBM (CUDA-graph
replay timed with CUDA events, max over ranks).  ``e2e`` = the same through
host buffers: pinned H2D copy of the step's input, the step, D2H copy of its
output, every step.  The weights (3.5 GB at TP=1, 0.44 GB per rank at TP=8)
exceed the 126 MB L2, so no flush is needed between steps.

``--impl reference`` times the reference's CPU path (the NumPy restatement in
oracle/, f32 dequantized weights, ranks run one after another as in
ie/parallel/tensor_parallel.py:65-73) on rank 0 with all host threads, on a
bounded sample of the same workload, scaled to the full step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "inference-engine_b200"))
sys.path.insert(0, str(REPO))

METRIC = "quant TP linear+allreduce % roofline; decode tok/s at TP=1/2/4/8"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--scheme", default="int4-g128")
    ap.add_argument("--unfused-norm", action="store_true",
                    help="run each rms_norm as its own kernel instead of inside the next GEMM")
    ap.add_argument("--sweep", action="store_true",
                    help="the isolated row-parallel GEMM + all-reduce sweep (one JSON line per "
                         "case) instead of the decode step")
    ap.add_argument("--sweep-m", default="1,8,64,512,4096,16384")
    ap.add_argument("--sweep-formats", default="int8,int4-g128,fp8")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return

        def read():
            for line in self.proc.stdout:
                self.rows.append([c.strip() for c in line.split(",")])

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm = [float(r[0]) for r in self.rows if len(r) >= 6 and r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if len(r) >= 6 and r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 6
                          for i in range(4) if r[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# the reference's CPU path (oracle port), bounded sample
# ---------------------------------------------------------------------------
def cpu_reference(args, world: int) -> dict:
    import numpy as np

    from oracle import tpq_oracle as o

    cores = os.cpu_count() or 1
    shape = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336)
    h, i = shape["hidden"], shape["inter"]
    q_out, kv_out = shape["heads"] * shape["head_dim"], shape["kv_heads"] * shape["head_dim"]
    rng = np.random.default_rng(0)
    # one layer of f32 dequantized weights (values do not change BLAS time)
    wq = rng.standard_normal((h, q_out), dtype=np.float32) * 0.02
    wk = rng.standard_normal((h, kv_out), dtype=np.float32) * 0.02
    wv = rng.standard_normal((h, kv_out), dtype=np.float32) * 0.02
    wo = rng.standard_normal((q_out, h), dtype=np.float32) * 0.02
    wg = rng.standard_normal((h, i), dtype=np.float32) * 0.02
    wu = rng.standard_normal((h, i), dtype=np.float32) * 0.02
    wd = rng.standard_normal((i, h), dtype=np.float32) * 0.02
    norm = np.ones(h, np.float32)
    x = rng.standard_normal((args.batch, h), dtype=np.float32)

    def layer(x):
        # ie/parallel/tensor_parallel.py:65-73 linear path, ranks in sequence
        parts = []
        for r in range(world):
            n = o.rms_norm(x, norm)
            a = n @ o.split_heads(wq, r, world, shape["heads"], shape["head_dim"])
            n @ o.split_heads(wk, r, world, shape["kv_heads"], shape["head_dim"])
            n @ o.split_heads(wv, r, world, shape["kv_heads"], shape["head_dim"])
            parts.append(a @ o.split_input_dim(wo, r, world))
        x = x + o.all_reduce(parts)
        parts = [o.sharded_mlp_partial(x, norm, wg, wu, wd, r, world) for r in range(world)]
        return x + o.all_reduce(parts)

    layer(x)
    reps, t0 = 0, time.perf_counter()
    while True:
        layer(x)
        reps += 1
        el = time.perf_counter() - t0
        if el > 10.0 or reps >= 50:
            break
    per_layer = el / reps
    step = per_layer * args.layers
    return {"value": args.batch / step, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": (f"{reps} passes over 1 of {args.layers} layers (Llama-3-8B shapes, "
                       f"batch {args.batch}, TP={world} ranks in sequence), NumPy f32 on "
                       f"dequantized weights, scaled x{args.layers}"),
            "ms_per_step": step * 1e3}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    base = cpu_reference(args, world)
    cfg = workload_config(args, world)
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PROFILE = REPO / "profiles" / "qgemm_tc_int4g128_b16_ncu_full.md"


def measured_traffic(args, kern_bytes: float, shape) -> tuple:
    """DRAM bytes (read + write) of one gate/up launch, from the committed ncu
    capture of the same kernel at TP=1, batch 16, int4-g128, scaled to this
    rank's launch by its algorithmic bytes (the traffic grows with the weight
    rows a rank owns).  None when the workload differs from the capture's."""
    if args.scheme != "int4-g128" or args.batch != 16:
        return None, "no capture for this scheme/batch"
    try:
        text = PROFILE.read_text()
    except OSError:
        return None, "profile summary missing"
    for line in text.splitlines():
        if "traffic_bytes_per_launch:" in line:
            field = line.split("traffic_bytes_per_launch:")[1].split()[0]
            measured = float(field.strip("`.,"))
            break
    else:
        return None, "profile summary has no traffic line"
    h, i = shape.hidden, shape.intermediate
    tp1 = (h * 2 * i / 2 + (h // 128) * 2 * i * 4) + args.batch * h * 2 + args.batch * i * 2
    return measured * kern_bytes / tp1, f"ncu dram__bytes_read+write, {PROFILE.name}"


def workload_config(args, world: int) -> dict:
    return {"workload": (f"Llama-3-8B-shaped decoder, quantized linear path of one decode step "
                         f"({args.layers} layers: qkv, o+allreduce, gate/up+SiLU, "
                         f"down+allreduce), {args.scheme} weights, bf16 activations"),
            "model": "llama3-8b-shaped (random init)", "scheme": args.scheme,
            "global_batch": args.batch, "seq_len": 1, "layers": args.layers,
            "parallelism": f"tp{world}",
            "l2": "weights per rank exceed the 126 MB L2; no flush between steps"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local: int) -> None:
    import torch

    torch.cuda.set_device(local)
    import torch.distributed as dist

    if world > 1:
        import datetime

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    from ie_tpq.comm import Communicator
    from ie_tpq.linear import qlinear
    from ie_tpq.sharding import Shard
    from ie_tpq.stack import LLAMA3_8B, LinearStack, layer_weight_bytes, synthetic_layer

    shape = LLAMA3_8B
    shard = Shard(rank, world)
    comm = None
    if world > 1:
        comm = Communicator(rank, world, max_bytes=max(args.batch * shape.hidden * 4, 1 << 20),
                            timeout_s=10.0)
    layers = [synthetic_layer(shape, args.scheme, shard, seed=1000 + li)
              for li in range(args.layers)]
    stack = LinearStack(shape, layers, args.batch, torch.bfloat16, comm=comm, world=world,
                        fuse_norm=not args.unfused_norm)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    stack.x_in.copy_(torch.randn(stack.x_in.shape, generator=gen, device="cuda"))
    stack.capture()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- resident-input throughput --------------------------------------
    for _ in range(args.warmup):
        stack.replay()
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    # keep the GPU under load while the sampler comes up (untimed)
    t_end = time.time() + 1.5
    while time.time() < t_end:
        for _ in range(20):
            stack.replay()
        torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        stack.replay()
    end.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    value = args.batch / (ms / 1e3)

    # ---- end to end through host buffers ---------------------------------
    x_host = torch.empty(stack.x_in.shape, dtype=stack.dtype).pin_memory()
    x_host.copy_(stack.x_in.cpu())
    out_host = torch.empty(stack.x_out.shape, dtype=stack.dtype).pin_memory()
    for _ in range(args.warmup):
        stack.run_host(x_host, out_host)
    torch.cuda.synchronize()
    barrier()
    start.record()
    for _ in range(args.steps):
        stack.run_host(x_host, out_host)
    end.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    if comm is not None:
        comm.check()

    # ---- dominant kernel: the gate/up launch of every layer, graph-replayed --
    wb = layer_weight_bytes(shape, args.scheme, world)
    h = torch.randn((args.batch, shape.hidden), generator=gen, device="cuda").to(torch.bfloat16)
    outs = [torch.empty((args.batch, L["gate_up"].out_features), dtype=torch.bfloat16,
                        device="cuda") for L in layers]
    for L, o_ in zip(layers, outs):
        qlinear(h, L["gate_up"], out=o_)
    torch.cuda.synchronize()
    kg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kg):
        for L, o_ in zip(layers, outs):
            qlinear(h, L["gate_up"], out=o_)
    kg.replay()
    torch.cuda.synchronize()
    reps = 5
    start.record()
    for _ in range(reps):
        kg.replay()
    end.record()
    torch.cuda.synchronize()
    kern_ms = start.elapsed_time(end) / (reps * len(layers))
    inter = 2 * shape.intermediate // world
    kern_bytes = wb["gate_up"] + args.batch * shape.hidden * 2 + args.batch * (inter // 2) * 2
    achieved = kern_bytes / (kern_ms / 1e3) / 1e9
    traffic, traffic_src = measured_traffic(args, kern_bytes, shape)
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        peak, peak_src = 6650.0, "fallback"

    if rank == 0:
        base = cpu_reference(args, world)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": workload_config(args, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "traffic_source": traffic_src,
                         "kernel": "qgemm_tc_kernel (tcgen05) gate/up, int4-g128, fused SiLU*up",
                         "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": kern_bytes,
                         "launch_us": kern_ms * 1e3},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": args.batch / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "gpu_launches": stack.launches_per_step * args.steps,
            "clocks": clocks,
            "weights_bytes_per_rank": args.layers * sum(wb.values()),
        }
        print(json.dumps(line), flush=True)
    barrier()
    del stack
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# isolated fused row-parallel GEMM + all-reduce sweep
# ---------------------------------------------------------------------------
SWEEP_KN = ((14336, 4096), (28672, 8192))
NVLINK_GBS = 770.0   # measured peer copy per direction on this pool's B200s


def sweep_bounds(scheme: str, m: int, k: int, n: int, world: int, w_bytes: float,
                 peaks: dict) -> dict:
    """Lower bounds of one rank's fused launch: HBM bytes (packed weights, x,
    out), tensor FLOPs and one-shot NVLink bytes ((world - 1) bf16 partials)."""
    hbm = w_bytes + m * k * 2 + m * n * 2
    flops = 2.0 * m * k * n
    nvl = (world - 1) * m * n * 2
    t = {"hbm": hbm / (peaks["hbm_gbs"] * 1e9),
         "tensor": flops / (peaks["bf16_tflops"] * 1e12),
         "nvlink": nvl / (NVLINK_GBS * 1e9)}
    bound = max(t, key=t.get)
    return {"bound": bound, "t_min_us": t[bound] * 1e6, "hbm_bytes": hbm, "flops": flops,
            "nvlink_bytes": nvl}


def run_sweep(args, rank: int, world: int, local: int) -> None:
    """The isolated row-parallel sweep: y = all_reduce(x_shard @ W_shard) for W [K, N] split by
    K over the ranks, fused (qlinear with comm=) against the unfused build
    (dequantize to bf16, cuBLAS GEMM, NCCL all-reduce), both timed with CUDA
    events and taken as the max over ranks."""
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    nccl = None
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        nccl = dist.new_group(backend="nccl")
    from ie_tpq.comm import Communicator
    from ie_tpq.linear import qlinear
    from ie_tpq.packed import quantize_on_device

    ms_list = [int(v) for v in args.sweep_m.split(",")]
    formats = args.sweep_formats.split(",")
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        peaks = {"hbm_gbs": float(peaks["hbm_gbs"]), "bf16_tflops": float(peaks["bf16_tflops"])}
        peak_src = "measured"
    except (OSError, KeyError, ValueError):
        peaks, peak_src = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"
    max_bytes = max(ms_list) * max(n for _, n in SWEEP_KN) * 4
    comm = Communicator(rank, world, max_bytes=max_bytes, timeout_s=10.0) if world > 1 else None

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, budget_ms: float = 60.0) -> float:
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        one = a.elapsed_time(b)
        reps = int(max(3, min(50, budget_ms / max(one, 1e-3))))
        reps = int(max_over_ranks(reps))   # every rank runs the same number of collectives
        if world > 1:
            dist.barrier()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b) / reps)

    gen = torch.Generator(device="cuda")
    for scheme in formats:
        for kk, n in SWEEP_KN:
            gen.manual_seed(0)
            full = torch.randn((kk, n), generator=gen, device="cuda") * 0.02
            k = kk // world
            w = quantize_on_device(full, scheme).slice_k(rank * k, (rank + 1) * k)
            del full
            torch.cuda.empty_cache()
            for m in ms_list:
                gen.manual_seed(1 + rank)
                x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
                out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")

                def fused():
                    qlinear(x, w, out=out, comm=comm)

                def unfused():
                    wd = w.dequantize("nk", torch.bfloat16)
                    y = x @ wd.t()
                    if world > 1:
                        dist.all_reduce(y, group=nccl)

                us_fused = timed(fused) * 1e3
                us_unfused = timed(unfused) * 1e3
                b = sweep_bounds(scheme, m, k, n, world, w.nbytes, peaks)
                if rank == 0:
                    print(json.dumps({
                        "sweep": "fused row-parallel quant GEMM + all-reduce", "scheme": scheme,
                        "K": kk, "N": n, "M": m, "tp": world, "k_per_rank": k,
                        "us_fused": us_fused, "us_unfused": us_unfused,
                        "speedup_vs_unfused": us_unfused / us_fused,
                        "roofline": {"bound": b["bound"], "t_min_us": b["t_min_us"],
                                     "frac": b["t_min_us"] / us_fused,
                                     "peak_source": peak_src,
                                     "nvlink_gbs": NVLINK_GBS},
                        "hbm_bytes": b["hbm_bytes"], "flops": b["flops"],
                        "nvlink_bytes": b["nvlink_bytes"]}), flush=True)
                del x, out
            del w
            torch.cuda.empty_cache()
    if comm is not None:
        comm.check()
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    rank, world, local = dist_env()
    if world == 1 and args.gpus > 1:
        print(json.dumps({"error": "launch with torchrun for --gpus > 1"}))
        sys.exit(2)
    if args.sweep:
        run_sweep(args, rank, world, local)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
