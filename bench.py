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
output, every step.  The weights (3.7 GB at TP=1, 0.46 GB per rank at TP=8)
exceed the 126 MB L2, so no flush is needed between steps.

Also in the line, all measured in the same run:
  * ``parity`` -- one eager pass of a layer at the bench's own shard shapes,
    every projection's output compared with the CPU oracle (rtol 2e-2 / atol
    2e-3) on a seeded subset of output columns, and the reduced outputs of all
    ranks compared bitwise;
  * ``dense_cublas`` -- the same step built the way the reference's GPU model
    runs it (ie/model/torch_transformer.py:15-29,36-38,60): dense bf16 weights
    resident on the device, torch matmul (cuBLAS), unfused norm / SiLU /
    residual, and an NCCL all-reduce per row-parallel layer at N > 1;
  * ``decode_batches`` -- the step at decode batches 1, 16, 64 and 256;
  * ``cpu_baseline`` -- the reference's NumPy path on the host cores.

``--impl reference`` times the reference's CPU path (the NumPy restatement in
oracle/, f32 dequantized weights, ranks run one after another as in
ie/parallel/tensor_parallel.py:65-73) on rank 0 with all host threads, on a
bounded sample of the same workload (whole layers), scaled to the full step.
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
RTOL, ATOL = 2e-2, 2e-3


# name -> (linear-path shape in ie_tpq.stack, model config in ie_tpq.model)
MODELS = {"llama3-8b": ("LLAMA3_8B", "LLAMA3_8B_CONFIG"),
          "llama3-70b": ("LLAMA3_70B", "LLAMA3_70B_CONFIG")}


def model_shape(args):
    import ie_tpq.stack as st

    return getattr(st, MODELS[args.model][0])


def model_config(args):
    import ie_tpq.model as md

    return getattr(md, MODELS[args.model][1])


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--model", choices=sorted(MODELS), default="llama3-8b",
                    help="decoder shape: Llama-3-8B (BASELINE config 3) or Llama-3-70B (config 4)")
    ap.add_argument("--layers", type=int, default=None, help="default: the model's")
    ap.add_argument("--scheme", default="int4-g128")
    ap.add_argument("--unfused-norm", action="store_true",
                    help="run each rms_norm as its own kernel instead of inside the next GEMM")
    ap.add_argument("--batches", default="1,16,64,256",
                    help="decode batches also timed (the decode_batches field); empty to skip")
    ap.add_argument("--no-dense", action="store_true", help="skip the dense cuBLAS comparator")
    ap.add_argument("--no-parity", action="store_true", help="skip the in-run parity check")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the model-level decode step (attention, lm_head, sampling)")
    ap.add_argument("--context", type=int, default=2048,
                    help="tokens already in every sequence's KV cache for the model decode step")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="wall-clock budget of the CPU baseline sample")
    ap.add_argument("--sweep", action="store_true",
                    help="the isolated row-parallel GEMM + all-reduce sweep (one JSON line per "
                         "case) instead of the decode step")
    ap.add_argument("--sweep-m", default="1,8,64,512,4096,16384")
    ap.add_argument("--allreduce", choices=["auto", "oneshot", "twoshot"], default="auto",
                    help="protocol of the fused all-reduce at N > 1 (the sweep times both)")
    ap.add_argument("--sweep-formats", default="int8,int4-g128,fp8,fp8-native")
    args = ap.parse_args()
    if args.layers is None:
        args.layers = {"llama3-8b": 32, "llama3-70b": 80}[args.model]
    return args


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
def cpu_reference(args, world: int, steps: int | None = None, warmup: int = 1) -> dict:
    """The reference's NumPy path for this workload on every host core: whole
    layers of ie/parallel/tensor_parallel.py:65-73 (ranks one after another),
    f32 dequantized weights.  One timed unit is one layer (a bounded sample of
    the step); ``steps`` units are timed after ``warmup`` (or, with steps None,
    as many as fit in ``--cpu-seconds``) and scaled to the full step.
    torchrun pins OMP_NUM_THREADS=1, so the BLAS pool is widened explicitly."""
    import numpy as np
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import tpq_oracle as o

    cores = os.cpu_count() or 1
    ms = model_shape(args)
    shape = dict(hidden=ms.hidden, heads=ms.heads, kv_heads=ms.kv_heads, head_dim=ms.head_dim,
                 inter=ms.intermediate)
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

    with threadpool_limits(limits=cores, user_api="blas"):
        threads = max((p.get("num_threads", 1) for p in threadpool_info()
                       if p.get("user_api") == "blas"), default=1)
        for _ in range(max(1, warmup)):
            layer(x)
        reps, t0 = 0, time.perf_counter()
        while True:
            layer(x)
            reps += 1
            el = time.perf_counter() - t0
            if steps is not None:
                if reps >= steps:
                    break
            elif el > args.cpu_seconds or reps >= 200:
                break
    per_layer = el / reps
    step = per_layer * args.layers
    return {"value": args.batch / step, "unit": UNIT, "cores": cores, "threads": threads,
            "kind": "port", "layers_timed": reps, "extrapolated_from_layers": 1,
            "sample": (f"{reps} passes over 1 of {args.layers} layers ({args.model} shapes, "
                       f"batch {args.batch}, TP={world} ranks in sequence), NumPy f32 on "
                       f"dequantized weights with {threads} BLAS threads on {cores} cores, "
                       f"scaled x{args.layers} to the step"),
            "ms_per_step": step * 1e3, "ms_timed": el * 1e3}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    base = cpu_reference(args, world, steps=args.steps, warmup=args.warmup)
    cfg = workload_config(args, world)
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "steps_note": (f"each step is a bounded sample of the decode step: one whole layer "
                           f"of the {args.layers}; the time per layer is scaled to the step"),
            "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "threads", "kind",
                                                  "sample", "extrapolated_from_layers",
                                                  "layers_timed")},
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PROFILE = REPO / "profiles" / "qgemm_tc_int4g128_b16_ncu_full.md"


# committed ncu captures of the gate/up launch at TP=1: (model, scheme, batch) -> summary
TRAFFIC_PROFILES = {
    ("llama3-8b", "int4-g128", 16): "qgemm_tc_int4g128_b16_ncu_full.md",
    ("llama3-70b", "fp8-native", 32): "qgemm_tc_fp8native_llama70b_b32_ncu_full.md",
}


def gate_up_tp1_bytes(scheme: str, batch: int, shape) -> float:
    """Algorithmic bytes of the TP=1 gate/up launch: packed weights and their
    tables, the activations and the SiLU*up output."""
    h, i = shape.hidden, shape.intermediate
    if scheme == "int4-g128":
        w = h * 2 * i / 2 + (h // 128) * 2 * i * 4
    else:   # fp8-native: one byte a weight, one f32 scale per output channel
        w = h * 2 * i + 2 * i * 4
    return w + batch * h * 2 + batch * i * 2


def measured_traffic(args, kern_bytes: float, shape) -> tuple:
    """DRAM bytes (read + write) of one gate/up launch, from the committed ncu
    capture of the same kernel at TP=1 and the same batch and scheme, scaled to
    this rank's launch by its algorithmic bytes (the traffic grows with the
    weight rows a rank owns).  None when no capture matches the workload."""
    name = TRAFFIC_PROFILES.get((args.model, args.scheme, args.batch))
    if name is None:
        return None, "no capture for this model/scheme/batch"
    path = PROFILE.parent / name
    try:
        text = path.read_text()
    except OSError:
        return None, "profile summary missing"
    for line in text.splitlines():
        if "traffic_bytes_per_launch:" in line:
            field = line.split("traffic_bytes_per_launch:")[1].split()[0]
            measured = float(field.strip("`.,"))
            break
    else:
        return None, "profile summary has no traffic line"
    tp1 = gate_up_tp1_bytes(args.scheme, args.batch, shape)
    return measured * kern_bytes / tp1, f"ncu dram__bytes_read+write, {path.name}"


def workload_config(args, world: int) -> dict:
    name = {"llama3-8b": "Llama-3-8B", "llama3-70b": "Llama-3-70B"}[args.model]
    acts = ("bf16 activations quantized per token to e4m3" if args.scheme == "fp8-native"
            else "bf16 activations")
    return {"workload": (f"{name}-shaped decoder, quantized linear path of one decode step "
                         f"({args.layers} layers: qkv, o+allreduce, gate/up+SiLU, "
                         f"down+allreduce), {args.scheme} weights, {acts}"),
            "model": f"{args.model}-shaped (random init)", "scheme": args.scheme,
            "global_batch": args.batch, "seq_len": 1, "layers": args.layers,
            "parallelism": f"tp{world}",
            "allreduce": args.allreduce if world > 1 else None,
            "l2": "weights per rank exceed the 126 MB L2; no flush between steps"}


# ---------------------------------------------------------------------------
# in-run parity at the bench's shard shapes
# ---------------------------------------------------------------------------
PARITY_COLS = 384


def parity_check(args, rank: int, world: int, shape, layer, seed: int, dist) -> dict:
    """One eager pass of a layer at this run's shard shapes, each projection
    compared with the CPU oracle on the GPU's own inputs to that projection.

    The oracle needs the f32 weights: rank 0 regenerates the layer's full
    weights with the seed ``synthetic_layer`` used and quantizes a seeded
    subset of PARITY_COLS output columns of each projection with the oracle's
    group-128 quantizer (group tables are per output column, so a column
    subset quantizes exactly as in the whole weight).  The reduced outputs of
    the row-parallel projections are compared bitwise across ranks."""
    import numpy as np
    import torch

    from ie_tpq.linear import fused_norm_ok, qlinear
    from ie_tpq.tensor_parallel import rms_norm
    from oracle import tpq_oracle as o

    h, inter = shape.hidden, shape.intermediate
    q_cols = shape.q_out // world
    native = args.scheme == "fp8-native"
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4242)
    x = torch.randn((args.batch, h), generator=gen, device="cuda").to(torch.bfloat16)
    norm = torch.ones(h, dtype=torch.float32, device="cuda")
    comm = layer.get("_comm")

    def norm_in(v, w):
        """(GEMM input, folded norm weight): the norm folded into the GEMM, or
        applied first (weights whose activations are quantized per token)."""
        return (v, norm) if fused_norm_ok(v, w) else (rms_norm(v, norm), None)

    first = layer["qkv"] if "qkv" in layer else layer["q"]
    h0, nw0 = norm_in(x, first)
    if "qkv" in layer:
        qkv = qlinear(h0, layer["qkv"], norm_weight=nw0)
    else:
        qkv = torch.cat([qlinear(h0, layer[n], norm_weight=nw0) for n in ("q", "k", "v")], 1)
    a = qkv[:, :q_cols].contiguous()
    x1 = qlinear(a, layer["o"], residual=x, comm=comm if world > 1 else None)
    h1, nw1 = norm_in(x1, layer["gate_up"])
    u = qlinear(h1, layer["gate_up"], norm_weight=nw1)
    x2 = qlinear(u, layer["down"], residual=x1, comm=comm if world > 1 else None)
    torch.cuda.synchronize()
    host = {k: v.float().cpu().numpy() for k, v in
            (("x", x), ("h0", h0), ("h1", h1), ("qkv", qkv), ("a", a), ("x1", x1), ("u", u),
             ("x2", x2))}
    fused0, fused1 = nw0 is not None, nw1 is not None
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, host)
    else:
        gathered = [host]
    if rank != 0:
        return {}
    bitwise = all(np.array_equal(g["x1"], gathered[0]["x1"]) and
                  np.array_equal(g["x2"], gathered[0]["x2"]) for g in gathered)
    # the layer's full f32 weights, in the order synthetic_layer draws them
    full = {}
    g2 = torch.Generator(device="cuda")
    g2.manual_seed(seed)
    for name, (k, n) in (("q", (h, shape.q_out)), ("k", (h, shape.kv_out)),
                         ("v", (h, shape.kv_out)), ("o", (shape.q_out, h)),
                         ("gate", (h, inter)), ("up", (h, inter)), ("down", (inter, h))):
        full[name] = torch.randn((k, n), generator=g2, device="cuda", dtype=torch.float32) * 0.02
    rng = np.random.default_rng(99)

    def deq_cols(w, cols, rows=None):
        """The oracle's dequantized weight on a subset of output columns (and
        a row shard): group-128 and per-N tables are per output column."""
        sub = w[:, torch.as_tensor(cols, device="cuda")].cpu().numpy()
        if args.scheme == "int4-g128":
            out = o.quantize_int4_group128(sub).dequantized()
        elif native:
            out = o.quantize_float(sub, *o.E4M3, axis=1).dequantized()
        else:
            raise ValueError("parity check implemented for int4-g128 and fp8-native")
        return out if rows is None else out[rows]

    def act(v):
        """A GEMM's activations as the kernel contracts them: per-token e4m3
        for fp8-native (o.quantize_activations_fp8), else as given."""
        return o.quantize_activations_fp8(v).dequantized() if native else v

    def row_parallel(parts, w, cols):
        """sum over ranks of act(x_r) @ W[rows of r] -- each rank quantizes its
        own K slice per token."""
        k = w.shape[0] // world
        wd = deq_cols(w, cols)
        return sum(act(xr) @ wd[r * k:(r + 1) * k] for r, xr in enumerate(parts))

    report, ok, worst = {}, bitwise, 0.0

    def compare(name, got, want):
        nonlocal ok, worst
        err = np.abs(got - want)
        fine = bool(np.all(err <= ATOL + RTOL * np.abs(want)))
        ok = ok and fine
        worst = max(worst, float(err.max()))
        report[name] = {"ok": fine, "max_abs": float(err.max()), "cols": int(got.shape[1])}

    heads = shape.heads
    hd = shape.head_dim
    xs = gathered[0]["x"]
    # the GEMM inputs: the oracle's rms_norm where the kernel folds it in, else
    # the normalised activations the GPU computed and fed to the GEMM
    n0 = act(o.rms_norm(xs, np.ones(h, np.float32)) if fused0 else gathered[0]["h0"])
    # qkv: rank r holds heads [r H/w, (r+1) H/w) of q, k and v
    q_all = np.concatenate([g["qkv"][:, :q_cols] for g in gathered], axis=1)
    cols = np.sort(rng.choice(shape.q_out, size=min(PARITY_COLS, shape.q_out), replace=False))
    compare("qkv(q heads)", q_all[:, cols], n0 @ deq_cols(full["q"], cols))
    # o: x1 = x + sum_r a_r @ Wo[rows of r]
    cols = np.sort(rng.choice(h, size=PARITY_COLS, replace=False))
    compare("o+allreduce+residual", gathered[0]["x1"][:, cols],
            xs[:, cols] + row_parallel([g["a"] for g in gathered], full["o"], cols))
    # gate/up: rank r holds columns [r I/w, (r+1) I/w) of both
    n1 = act(o.rms_norm(gathered[0]["x1"], np.ones(h, np.float32)) if fused1
             else gathered[0]["h1"])
    u_all = np.concatenate([g["u"] for g in gathered], axis=1)
    cols = np.sort(rng.choice(inter, size=PARITY_COLS, replace=False))
    want = o.silu(n1 @ deq_cols(full["gate"], cols)) * (n1 @ deq_cols(full["up"], cols))
    compare("gate/up+silu", u_all[:, cols], want)
    cols = np.sort(rng.choice(h, size=PARITY_COLS, replace=False))
    compare("down+allreduce+residual", gathered[0]["x2"][:, cols],
            gathered[0]["x1"][:, cols] + row_parallel([g["u"] for g in gathered], full["down"],
                                                      cols))
    del full
    torch.cuda.empty_cache()
    return {"ok": ok, "max_abs": worst, "ranks_bitwise_equal": bitwise, "rtol": RTOL,
            "atol": ATOL,
            "oracle": ("oracle/tpq_oracle.py " +
                       ("per-token e4m3 activations (quantize_activations_fp8) and per-N e4m3 "
                        "weights" if native else "int4 group-128") + ", f32 dequant-matmul"),
            "shapes": {"qkv": [h, (shape.q_out + 2 * shape.kv_out) // world],
                       "o": [shape.q_out // world, h], "gate_up": [h, 2 * inter // world],
                       "down": [inter // world, h]},
            "tokens": args.batch, "projections": report}


# ---------------------------------------------------------------------------
# the comparator: dense bf16 weights, cuBLAS, NCCL (the reference's GPU model)
# ---------------------------------------------------------------------------
def dense_step(args, world: int, shape, steps: int, warmup: int, nccl, max_over_ranks, barrier):
    """The decode step's linear path as TorchTransformer runs it: dense bf16
    weights resident on the device, ``x @ W`` on cuBLAS for every projection,
    rms_norm / SiLU*up / residual as separate torch ops, and an NCCL all-reduce
    after each row-parallel projection at N > 1.  Weight values do not change
    cuBLAS time, so they are random bf16 drawn on the device.  Returns ms per
    step (CUDA-graph replay, max over ranks)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    h, inter = shape.hidden, shape.intermediate
    qkv_n = (shape.q_out + 2 * shape.kv_out) // world
    q_cols = shape.q_out // world
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    mk = lambda n, k: (torch.randn((n, k), generator=gen, device="cuda",
                                   dtype=torch.float32) * 0.02).to(torch.bfloat16)
    layers = [{"qkv": mk(qkv_n, h), "o": mk(h, q_cols), "gu": mk(2 * inter // world, h),
               "down": mk(h, inter // world)} for _ in range(args.layers)]
    norm = torch.ones(h, dtype=torch.bfloat16, device="cuda")
    x_in = torch.randn((args.batch, h), generator=gen, device="cuda").to(torch.bfloat16)
    x_out = torch.empty_like(x_in)
    half = inter // world

    def step():
        x = x_in
        for L in layers:
            n = F.rms_norm(x, (h,), norm, 1e-6)
            qkv = n @ L["qkv"].t()
            o_ = qkv[:, :q_cols] @ L["o"].t()
            if world > 1:
                dist.all_reduce(o_, group=nccl)
            x = x + o_
            n = F.rms_norm(x, (h,), norm, 1e-6)
            gu = n @ L["gu"].t()
            u = F.silu(gu[:, :half]) * gu[:, half:]
            d = u @ L["down"].t()
            if world > 1:
                dist.all_reduce(d, group=nccl)
            x = x + d
        x_out.copy_(x)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(a.elapsed_time(b) / steps)
    wbytes = sum(t.numel() * 2 for L in layers for t in L.values())
    del g, layers
    torch.cuda.empty_cache()
    return ms, wbytes


# ---------------------------------------------------------------------------
# model-level decode step (decode at a 2048-token context)
# ---------------------------------------------------------------------------
MODEL_BLOCK = 256   # KV block size: flash-attn's paged kernels take multiples of 256


def _decode_inputs(batch: int, context: int, seed: int):
    """Static device inputs of one decode step: every sequence holds `context`
    tokens (positions 0 .. context-2 cached, the new token at context-1) in its
    own run of KV blocks."""
    import torch

    per = (context + MODEL_BLOCK - 1) // MODEL_BLOCK
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    tables = torch.arange(batch * per, device="cuda", dtype=torch.long).reshape(batch, per)
    pos = context - 1
    return {
        "tokens": torch.randint(0, 128256, (batch,), generator=gen, device="cuda"),
        "positions": torch.full((batch,), pos, dtype=torch.long, device="cuda"),
        "tables": tables,
        "slots": tables[:, pos // MODEL_BLOCK] * MODEL_BLOCK + pos % MODEL_BLOCK,
        "context_lens": torch.full((batch,), context, dtype=torch.int32, device="cuda"),
        "num_blocks": batch * per,
    }


def _graph_ms(step, steps: int, warmup: int, barrier, max_over_ranks):
    """CUDA-graph one call of `step`, replay it: ms per replay (max over ranks)."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    ms = timed_replays(g.replay, steps, warmup, barrier, max_over_ranks)
    del g
    return ms


def model_decode(args, rank: int, world: int, comm, nccl, barrier, max_over_ranks) -> dict:
    """One decode step of the whole Llama-3-8B-shaped model at `args.batch`
    sequences of `args.context` tokens, through ``QuantizedTransformer.run``
    (the Engine-protocol model: embedding, per layer qkv / RoPE / KV write /
    flash-attn paged decode / o + fused all-reduce / gate-up / down + fused
    all-reduce, final norm) and ``greedy_on_device`` (vocab-parallel lm_head,
    argmax), with each step's tokens fed back as the next step's input.  The
    comparator is the same step as the reference's TorchTransformer runs it on
    the GPU: dense bf16 weights, cuBLAS matmuls, the same RoPE / KV write /
    flash-attn calls, NCCL all-reduces at N > 1."""
    import torch

    from ie_tpq.decode import Layout
    from ie_tpq.model import QuantizedTransformer, synthetic_source
    from ie_tpq.sharding import Shard

    cfg = model_config(args)
    if args.layers != cfg.num_layers:
        from dataclasses import replace

        cfg = replace(cfg, num_layers=args.layers)
    batch = args.batch
    src = synthetic_source(cfg, args.scheme, seed=3)
    model = QuantizedTransformer(src, scheme=args.scheme, shard=Shard(rank, world),
                                 comm=comm if world > 1 else None, dtype=torch.bfloat16)
    del src
    torch.cuda.empty_cache()
    inp = _decode_inputs(batch, args.context, seed=11)
    k_caches, v_caches = model.allocate_caches(inp["num_blocks"], MODEL_BLOCK)
    plan = {"flash": True, "scale": cfg.head_dim ** -0.5, "slots": inp["slots"],
            "context_lens": inp["context_lens"], "cu_q": None, "cu_k": None,
            "paged_tables": None, "tables32": inp["tables"].to(torch.int32)}
    layout = Layout([0] * batch, [args.context - 1] * batch, [0] * batch,
                    [args.context] * batch, [1] * batch, [[0]] * batch, False)
    tokens = inp["tokens"]

    def ours():
        h = model.run(tokens, inp["positions"], inp["tables"], plan, layout, k_caches,
                      v_caches, MODEL_BLOCK)
        tokens.copy_(model.greedy_on_device(h))

    steps = max(20, min(args.steps, 200))
    ms = _graph_ms(ours, steps, 3, barrier, max_over_ranks)
    def packed_bytes(w):
        return (w.codes.numel() + w.scale.numel() * w.scale.element_size() +
                (w.zero.numel() * w.zero.element_size() if w.zero is not None else 0))

    wbytes = sum(packed_bytes(w) for a, m in zip(model.attn, model.mlp)
                 for w in ([a.qkv] if a.qkv is not None else [a.q_proj, a.k_proj, a.v_proj]) +
                 [a.o_proj, m.gate_up, m.down])
    out = {"tok_s": batch / (ms / 1e3), "ms_per_step": ms, "batch": batch,
           "context": args.context, "kv_block": MODEL_BLOCK, "steps": steps,
           "linear_weight_bytes_per_rank": wbytes}
    del model
    torch.cuda.empty_cache()
    if not args.no_dense:
        dms = _dense_model_ms(args, cfg, world, rank, nccl, inp, k_caches, v_caches, steps,
                              barrier, max_over_ranks)
        out["dense_cublas"] = {"tok_s": batch / (dms / 1e3), "ms_per_step": dms,
                               "speedup_of_ours": dms / ms}
    del k_caches, v_caches
    torch.cuda.empty_cache()
    return out


def _dense_model_ms(args, cfg, world, rank, nccl, inp, k_caches, v_caches, steps, barrier,
                    max_over_ranks) -> float:
    """The decode step of ``model_decode`` with dense bf16 weights (the
    reference's TorchTransformer on the GPU: ie/model/torch_transformer.py:31-63,
    ie/kernels/torch_backend.py:103-127), this rank's TP shards."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from ie_tpq.attention import apply_rope, flash_decode, write_kv
    from ie_tpq.model import rope_tables_on_device

    h, inter = cfg.hidden_size, cfg.intermediate_size // world
    hd = cfg.head_dim
    nh, nkv = cfg.num_heads // world, cfg.num_kv_heads // world
    vocab = cfg.vocab_size // world
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    mk = lambda n, k: (torch.randn((n, k), generator=gen, device="cuda",
                                   dtype=torch.float32) * 0.02).to(torch.bfloat16)
    layers = [{"qkv": mk((nh + 2 * nkv) * hd, h), "o": mk(h, nh * hd), "gu": mk(2 * inter, h),
               "down": mk(h, inter)} for _ in range(cfg.num_layers)]
    emb = mk(cfg.vocab_size, h)
    lm_head = mk(vocab, h)
    norm = torch.ones(h, dtype=torch.bfloat16, device="cuda")
    cos, sin = rope_tables_on_device(cfg.max_position, hd, cfg.rope_base, "cuda")
    tokens = inp["tokens"]
    scale = hd ** -0.5

    def step():
        x = emb.index_select(0, tokens)
        for L, kc, vc in zip(layers, k_caches, v_caches):
            n = F.rms_norm(x, (h,), norm, cfg.norm_eps)
            qkv = n @ L["qkv"].t()
            q = qkv[:, :nh * hd].reshape(-1, nh, hd)
            k = qkv[:, nh * hd:(nh + nkv) * hd].reshape(-1, nkv, hd)
            v = qkv[:, (nh + nkv) * hd:].reshape(-1, nkv, hd)
            q = apply_rope(q, inp["positions"], cos, sin)
            k = apply_rope(k, inp["positions"], cos, sin)
            write_kv(k, v, kc, vc, inp["slots"])
            a = flash_decode(q, kc, vc, inp["tables"].int(), inp["context_lens"], MODEL_BLOCK,
                             scale).reshape(-1, nh * hd)
            o_ = a @ L["o"].t()
            if world > 1:
                dist.all_reduce(o_, group=nccl)
            x = x + o_
            n = F.rms_norm(x, (h,), norm, cfg.norm_eps)
            gu = n @ L["gu"].t()
            d = (F.silu(gu[:, :inter]) * gu[:, inter:]) @ L["down"].t()
            if world > 1:
                dist.all_reduce(d, group=nccl)
            x = x + d
        x = F.rms_norm(x, (h,), norm, cfg.norm_eps)
        local = (x @ lm_head.t()).float()
        idx = local.argmax(dim=-1)
        if world > 1:
            buf = torch.zeros((world, 2, x.shape[0]), dtype=torch.float32, device="cuda")
            buf[rank, 0] = local.gather(1, idx[:, None]).squeeze(1)
            buf[rank, 1] = (idx + rank * vocab).float()
            dist.all_reduce(buf, group=nccl)
            idx = buf[:, 1].gather(0, buf[:, 0].argmax(dim=0)[None]).squeeze(0).long()
        tokens.copy_(idx)

    ms = _graph_ms(step, steps, 3, barrier, max_over_ranks)
    del layers, emb, lm_head
    torch.cuda.empty_cache()
    return ms


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def timed_replays(fn, steps: int, warmup: int, barrier, max_over_ranks):
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    barrier()
    return max_over_ranks(a.elapsed_time(b) / steps)


def run_ours(args, rank: int, world: int, local: int) -> None:
    import torch

    torch.cuda.set_device(local)
    import torch.distributed as dist

    nccl = None
    if world > 1:
        import datetime

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
        if not args.no_dense:
            nccl = dist.new_group(backend="nccl")
    from ie_tpq.comm import Communicator
    from ie_tpq.linear import qlinear
    from ie_tpq.sharding import Shard
    from ie_tpq.stack import LinearStack, layer_weight_bytes, synthetic_layer

    shape = model_shape(args)
    shard = Shard(rank, world)
    comm = None
    if world > 1:
        comm = Communicator(rank, world, max_bytes=max(max(args.batch, 256) * shape.hidden * 4,
                                                       1 << 20), timeout_s=10.0,
                            algo=ALLREDUCE_ALGOS[args.allreduce])
    layers = [synthetic_layer(shape, args.scheme, shard, seed=1000 + li)
              for li in range(args.layers)]
    stack = LinearStack(shape, layers, args.batch, torch.bfloat16, comm=comm, world=world,
                        fuse_norm=not args.unfused_norm)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    stack.x_in.copy_(torch.randn(stack.x_in.shape, generator=gen, device="cuda"))
    stack.capture()
    launches_per_step = stack.launches_per_step   # this library's kernels per step

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
    e2e_ms = timed_replays(lambda: stack.run_host(x_host, out_host), args.steps, args.warmup,
                           barrier, max_over_ranks)
    if comm is not None:
        comm.check()

    # ---- the step at other decode batches ----------------------------------
    batches = {}
    for b in [int(v) for v in args.batches.split(",") if v.strip()]:
        if b == args.batch:
            batches[str(b)] = {"tok_s": value, "ms_per_step": ms}
            continue
        st = LinearStack(shape, layers, b, torch.bfloat16, comm=comm, world=world,
                         fuse_norm=not args.unfused_norm)
        st.x_in.copy_(torch.randn(st.x_in.shape, generator=gen, device="cuda"))
        st.capture()
        reps = max(20, min(args.steps, 200))
        bms = timed_replays(st.replay, reps, 3, barrier, max_over_ranks)
        batches[str(b)] = {"tok_s": b / (bms / 1e3), "ms_per_step": bms, "steps": reps}
        del st
    torch.cuda.empty_cache()

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
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        peak, peak_src = 6650.0, "fallback"
    del kg, outs
    torch.cuda.empty_cache()

    # ---- parity of one layer at these shard shapes ---------------------------
    parity = None
    if not args.no_parity:
        layer0 = dict(layers[0])
        layer0["_comm"] = comm
        parity = parity_check(args, rank, world, shape, layer0, 1000, dist)

    # ---- the dense cuBLAS (+ NCCL) comparator --------------------------------
    dense = None
    weight_bytes = args.layers * sum(wb.values())
    if not args.no_dense:
        del stack
        layers.clear()
        torch.cuda.empty_cache()
        dms, dbytes = dense_step(args, world, shape, max(20, min(args.steps, 300)), 5, nccl,
                                 max_over_ranks, barrier)
        dense = {"value": args.batch / (dms / 1e3), "unit": UNIT, "ms_per_step": dms,
                 "speedup_of_ours": value / (args.batch / (dms / 1e3)),
                 "weights_bytes_per_rank": dbytes,
                 "what": ("dense bf16 weights resident, torch matmul (cuBLAS), unfused "
                          "rms_norm/SiLU/residual" + (", NCCL all-reduce" if world > 1 else "") +
                          "; CUDA graph, CUDA events, max over ranks")}

    # ---- the whole model's decode step (attention, lm_head, sampling) --------
    model = None
    if not args.no_model:
        stack = None   # release the linear-path stack (if the dense arm has not)
        layers.clear()
        torch.cuda.empty_cache()
        model = model_decode(args, rank, world, comm, nccl, barrier, max_over_ranks)

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
                         "kernel": f"qgemm_tc_kernel (tcgen05) gate/up, {args.scheme}, fused SiLU*up",
                         "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": kern_bytes,
                         "launch_us": kern_ms * 1e3,
                         "step_weight_bytes_per_rank": weight_bytes,
                         "step_frac": weight_bytes / (ms / 1e3) / 1e9 / peak},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "threads", "kind",
                                                  "sample", "extrapolated_from_layers",
                                                  "layers_timed")},
            "e2e": {"value": args.batch / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "parity": parity,
            "dense_cublas": dense,
            "model_decode": model,
            "decode_batches": batches,
            "weights_bytes_per_rank": weight_bytes,
        }
        print(json.dumps(line), flush=True)
    barrier()
    if comm is not None:
        comm.close()
    if world > 1:
        if nccl is not None:
            dist.destroy_process_group(nccl)
        dist.destroy_process_group()



# ---------------------------------------------------------------------------
# isolated fused row-parallel GEMM + all-reduce sweep
# ---------------------------------------------------------------------------
SWEEP_KN = ((14336, 4096), (28672, 8192))
ALLREDUCE_ALGOS = {"auto": 0, "oneshot": 1, "twoshot": 2}   # ie_tpq.comm.AR_*
NVLINK_GBS = 770.0   # measured B200 peer copy bandwidth, GB/s per direction


def sweep_bounds(scheme: str, m: int, k: int, n: int, world: int, w_bytes: float,
                 peaks: dict) -> dict:
    """Lower bounds of one rank's fused launch: HBM bytes (packed weights, x,
    out), tensor FLOPs and one-shot NVLink bytes ((world - 1) bf16 partials).
    The tensor bound is the measured bf16 GEMM rate, or twice it for the
    native fp8 contraction (B200's dense fp8 rate is twice its bf16 rate)."""
    hbm = w_bytes + m * k * 2 + m * n * 2
    flops = 2.0 * m * k * n
    nvl = (world - 1) * m * n * 2
    tensor_peak = peaks["bf16_tflops"] * (2.0 if scheme == "fp8-native" else 1.0)
    t = {"hbm": hbm / (peaks["hbm_gbs"] * 1e9),
         "tensor": flops / (tensor_peak * 1e12),
         "nvlink": nvl / (NVLINK_GBS * 1e9)}
    bound = max(t, key=t.get)
    return {"bound": bound, "t_min_us": t[bound] * 1e6, "hbm_bytes": hbm, "flops": flops,
            "nvlink_bytes": nvl}


def _lib_act_fp8() -> int:
    from ie_tpq import _lib

    return _lib.IE_ACT_FP8_TOKEN


def run_sweep(args, rank: int, world: int, local: int) -> None:
    """The isolated row-parallel sweep: y = all_reduce(x_shard @ W_shard) for W [K, N] split by
    K over the ranks, fused (qlinear with comm=) against two unfused builds,
    all timed as CUDA-graph replays with CUDA events and taken as the max
    over ranks:
      * ``us_unfused`` -- dequantize the shard to bf16 on every call, cuBLAS GEMM,
        NCCL all-reduce (a quantized model served without a fused kernel);
      * ``us_dense`` -- the dequantized bf16 shard kept resident (the reference's
        own GPU model, ie/model/torch_transformer.py:15-29), cuBLAS GEMM, NCCL."""
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    nccl = None
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        nccl = dist.new_group(backend="nccl")
    from ie_tpq.comm import AR_ONESHOT, AR_TWOSHOT, Communicator, resolve_algo
    from ie_tpq.linear import qlinear
    from ie_tpq.packed import quantize_on_device

    def resolve_name(world_, m_, n_):
        tiles = -(-n_ // 128) * -(-m_ // 256)
        return "oneshot" if resolve_algo(world_, tiles, m_ * n_) == AR_ONESHOT else "twoshot"

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

    inner = 8   # calls per captured graph

    def timed(fn, budget_ms: float = 60.0) -> float:
        """ms per call of ``fn``: a CUDA graph of ``inner`` consecutive calls
        is replayed, so host launch costs do not enter small cases while
        consecutive kernels still overlap as in a model's step graph
        (programmatic launch); max over ranks.  Eager calls if capture fails."""
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        per = 1
        try:
            g = torch.cuda.CUDAGraph()
            s_ = torch.cuda.Stream()
            s_.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s_):
                fn()
            torch.cuda.current_stream().wait_stream(s_)
            torch.cuda.synchronize()
            with torch.cuda.graph(g):
                for _ in range(inner):
                    fn()
            g.replay()
            torch.cuda.synchronize()
            fn, per = g.replay, inner
        except RuntimeError:
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
        return max_over_ranks(a.elapsed_time(b) / (reps * per))

    gen = torch.Generator(device="cuda")
    for scheme in formats:
        for kk, n in SWEEP_KN:
            gen.manual_seed(0)
            full = torch.randn((kk, n), generator=gen, device="cuda") * 0.02
            k = kk // world
            # fp8-native: per-N fp8 weights and per-token fp8 activations on
            # the tensor cores (act_quant); the others dequantize the weight
            native = scheme == "fp8-native"
            act = _lib_act_fp8() if native else 0
            w = quantize_on_device(full, "fp8" if native else scheme,
                                   axis=1 if native else 0).slice_k(rank * k, (rank + 1) * k)
            del full
            # the dense comparator keeps the dequantized bf16 shard resident
            w_dense = w.dequantize("nk", torch.bfloat16)
            torch.cuda.empty_cache()
            for m in ms_list:
                gen.manual_seed(1 + rank)
                x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
                out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")

                def fused(algo=None):
                    qlinear(x, w, out=out, comm=comm, act_quant=act, reduce_algo=algo)

                def unfused():
                    wd = w.dequantize("nk", torch.bfloat16)
                    y = x @ wd.t()
                    if world > 1:
                        dist.all_reduce(y, group=nccl)

                def dense():
                    y = x @ w_dense.t()
                    if world > 1:
                        dist.all_reduce(y, group=nccl)

                us_fused = timed(fused) * 1e3
                protocols = {}
                if world > 1:
                    # both protocols, and the NVLink bytes each sends per rank
                    # (f32 partials; two-shot's finished tiles also f32)
                    for name, code in (("oneshot", AR_ONESHOT), ("twoshot", AR_TWOSHOT)):
                        us = timed(lambda: fused(code)) * 1e3
                        tiles = -(-n // 128) * -(-m // 256)
                        used = resolve_algo(world, tiles, m * n, code)
                        sent = (m * n * 4 * (world - 1) if used == AR_ONESHOT
                                else m * n * 8 * (world - 1) / world)
                        protocols[name] = {"us": us, "ran": "oneshot" if used == AR_ONESHOT
                                           else "twoshot", "nvlink_bytes_sent": sent,
                                           "nvlink_gbs": sent / (us * 1e3)}
                us_unfused = timed(unfused) * 1e3
                us_dense = timed(dense) * 1e3
                b = sweep_bounds(scheme, m, k, n, world, w.nbytes, peaks)
                if rank == 0:
                    print(json.dumps({
                        "sweep": "fused row-parallel quant GEMM + all-reduce", "scheme": scheme,
                        "K": kk, "N": n, "M": m, "tp": world, "k_per_rank": k,
                        "us_fused": us_fused, "us_unfused": us_unfused, "us_dense": us_dense,
                        "speedup_vs_unfused": us_unfused / us_fused,
                        "speedup_vs_dense": us_dense / us_fused,
                        "roofline": {"bound": b["bound"], "t_min_us": b["t_min_us"],
                                     "frac": b["t_min_us"] / us_fused,
                                     "peak_source": peak_src,
                                     "nvlink_gbs": NVLINK_GBS},
                        "hbm_bytes": b["hbm_bytes"], "flops": b["flops"],
                        "nvlink_bytes": b["nvlink_bytes"],
                        "allreduce_auto": protocols and resolve_name(world, m, n),
                        "protocols": protocols}), flush=True)
                del x, out
            del w, w_dense
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
