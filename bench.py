#!/usr/bin/env python
"""TTCLayer forward+backward throughput (tokens/s) on B200 -- BASELINE.json's metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl cuda|reference]

One step = TTCLayer forward + backward on one batch of the chosen config, rows read as
[B, L*H, in_dim], with the parameter gradients and dx of the whole batch (gradient
accumulation over row micro-batches where one call's activations would not fit).  Default:
config 3 per GPU (bf16 activations, fp32 solver, x[8,4096,32,128], h_dim 32, T 128), which
is also config 5's per-GPU shard at 8 GPUs.  At N > 1 (torchrun) every rank runs the same
per-GPU batch on its own data and the parameter gradients are all-reduced (NCCL) inside the
step: weak scaling, so N = 8 runs config 5's global batch of 64 sequences.  ``--config 5``
instead splits config 5's global batch over the N GPUs (strong scaling, as BASELINE.json
defines it).  Rank 0 prints one JSON line.

``--impl reference`` times the reference's CPU path, its own ``TTCLayer(solver_impl="riccati")``
forward + autograd backward from the unmodified install in baseline/_ref (fla's Triton l2norm
replaced by its formula on CPU tensors; the oracle's restatement when that install is absent),
fp32, all host threads, on a row sample of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (REPO, os.path.join(REPO, "ttc-net_b200"), os.path.join(REPO, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from ttc_cases import CONFIGS, layer_input, layer_weights  # noqa: E402

METRIC = "TTCLayer fwd+bwd tokens/sec"
L2_BYTES = 126 * 2**20
SM_COUNT_B200 = 148
FP32_LANES_PER_SM = 128


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--chunk-rows", type=int, default=0,
                    help="rows (of B*L*H) per layer call inside a step (0: TTCLayer.rows_per_call)")
    ap.add_argument("--batch", type=int, default=0,
                    help="sequences per GPU (0: the config's B); smaller batches for ncu captures")
    ap.add_argument("--seq-len", type=int, default=0,
                    help="positions per sequence (0: the config's L); a fraction of a config's rows "
                         "(rows are independent, so tokens/s carries over)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--solver", default="cuda", choices=["cuda", "kkt"],
                    help="the layer's solver_impl (kkt: the reference's two-problem backward on the GPU)")
    ap.add_argument("--workload", default="layer", choices=["layer", "traj"],
                    help="layer: the headline TTCLayer step; traj: closed-loop trajectories "
                         "(lqr_trajectory) of the config's solver inputs, one GPU")
    ap.add_argument("--traj-rows", type=int, default=0,
                    help="rows of the trajectory workload (0: the config's per-GPU batch)")
    return ap.parse_args(argv)


# ------------------------------------------------------------------------- FLOP model
def solver_flops(cfg):
    """Algorithmic FLOPs per LQR problem (2 per FMA; recompute not counted)."""
    d = du = cfg.h_dim
    T = cfg.T
    fwd = T * 4 * d * d * du + (T - 1) * 2 * d**3 + (2 / 3) * d**3 + 2 * d**3 + 4 * d * d + 4 * d * du
    bwd = T * (8 * d * d + 12 * d * du) + 2 * d * du + 2 * d * d
    return fwd, bwd


# ------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: str, startup_s: float = 30.0):
        self.gpu = gpu
        self.startup_s = startup_s
        self.proc = None
        self.lines = []
        self.err = ""
        self.first = threading.Event()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi needs up to seconds to initialise on a many-GPU box; the timed
            # region starts only after its first sample so that short runs are covered.
            self.first.wait(self.startup_s)
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self.first.set()
        self.first.set()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)
            try:
                self.err = (self.proc.stderr.read() or "").strip().splitlines()[-1:]
            except (OSError, ValueError):
                self.err = []

    def summary(self):
        if not self.lines:
            why = "; ".join(self.err) if self.err else "no sample"
            return {"sm_mhz": None, "sm_max_mhz": None,
                    "reasons": [f"nvidia-smi unavailable ({why}, -i {self.gpu})"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_selector(local: int) -> str:
    """nvidia-smi -i argument for this process's GPU: its UUID (immune to
    CUDA_VISIBLE_DEVICES renumbering), else the visible-device entry, else the index."""
    try:
        u = str(torch.cuda.get_device_properties(local).uuid)
        if u:
            return u if u.startswith("GPU-") else "GPU-" + u
    except (AttributeError, RuntimeError):
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        return vis.split(",")[local].strip()
    return str(local)


# ------------------------------------------------------------------------- setup
def dist_setup(ngpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != ngpus:
        raise SystemExit(f"--gpus {ngpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def make_layer(cfg, device, dtype, solver="cuda"):
    from ttc_b200 import TTCLayer
    layer = TTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                     solver_impl=solver)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    return layer.to(device=device, dtype=dtype)


def run_step(layer, x, dy, T, chunk, world, reducer=None):
    """One fwd+bwd over the batch: TTCLayer.forward_backward (row micro-batches of `chunk`
    rows, gradient accumulation), the parameter gradients and dx, as the end-to-end step and
    the CPU baseline compute them.  At N > 1 `reducer` (an OverlappedGradAllReduce) all-reduces
    each parameter gradient as soon as the last micro-batch's backward has completed it."""
    layer.zero_grad(set_to_none=True)
    x.grad = None
    layer.forward_backward(x, dy, T, rows=chunk, before_last_backward=reducer.arm if reducer else None)
    if reducer is not None:
        reducer.wait()


# ------------------------------------------------------------------------- CPU legs
REFERENCE_INSTALL = os.path.join(REPO, "baseline", "_ref")


def reference_cpu_layer(cfg):
    """The reference's own TTCLayer(solver_impl="riccati") from its unmodified install in
    baseline/_ref (pip install --target), with fla's l2norm -- a Triton wrapper that does not
    run on CPU tensors -- replaced by its formula x / sqrt(sum x^2 + 1e-6) in fp32
    (fla/modules/l2norm.py:42); None when the install is absent.  Returns (layer, kind)."""
    if not os.path.isdir(os.path.join(REFERENCE_INSTALL, "ttc")):
        return None
    if REFERENCE_INSTALL not in sys.path:
        sys.path.insert(0, REFERENCE_INSTALL)
    try:
        import ttc.layers.ttc_layer as ref_mod
    except Exception:  # noqa: BLE001 - any import failure means: use the port
        return None

    def l2norm_cpu(x, eps=1e-6):
        xf = x.float()
        return (xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)

    ref_mod.l2norm = l2norm_cpu
    return ref_mod.TTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                            solver_impl="riccati")


def cpu_sample(cfg, target_s, threads, rows=None):
    """Reference algorithm on the host: the riccati layer fwd + autograd bwd (the reference's
    own TTCLayer from baseline/_ref when installed, else the oracle's restatement of it) on a
    row sample sized to ~target_s seconds (or of `rows` rows).  Returns (tokens/s, rows,
    seconds, kind) with kind "reference" or "port"."""
    torch.set_num_threads(threads)
    layer, kind = reference_cpu_layer(cfg), "reference"
    if layer is None:
        from oracle import ttc_oracle as O
        layer, kind = O.TTCLayerOracle(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                                       solver_impl="riccati"), "port"
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})

    def once(rows):
        x_np, dy_np = layer_input(cfg, rows, seed=cfg.seed + 77)
        x = torch.from_numpy(x_np)[None].requires_grad_(cfg.backward)
        t0 = time.perf_counter()
        y = layer(x, T=cfg.T)
        if cfg.backward:
            y.backward(torch.from_numpy(dy_np)[None])
        return time.perf_counter() - t0

    if rows is not None:
        dt = once(rows)
        return (rows / cfg.H) / dt, rows, dt, kind
    # A tiny probe is dominated by per-step Python overhead and overestimates the cost of a
    # row; one more rescale from the first real sample brings the sample to ~target_s.
    probe = max(1, cfg.H // 8)
    t = once(probe)
    rows = int(max(probe, min(cfg.rows, probe * target_s / max(t, 1e-6))))
    dt = once(rows)
    if dt < 0.5 * target_s and rows < cfg.rows:
        rows = int(min(cfg.rows, rows * target_s / max(dt, 1e-6)))
        dt = once(rows)
    return (rows / cfg.H) / dt, rows, dt, kind


def reference_arm(args, cfg):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    budget = 150.0 / max(1, args.steps + args.warmup)
    vals = []
    rows_used = None
    kind = "port"
    for k in range(args.warmup + args.steps):
        v, rows_used, _, kind = cpu_sample(cfg, budget, threads, rows_used)
        if k >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    what = ("the reference's TTCLayer from baseline/_ref, fla l2norm as its formula" if kind == "reference"
            else "oracle port")
    sample = (f"{rows_used} of {cfg.rows} rows per step ({cfg.name}: riccati fwd + autograd "
              f"bwd, fp32, {what})")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * (rows_used / cfg.H) / value, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {**workload_config(cfg, world, args, chunk=None),
                   "solver_impl": f"riccati ({what}, CPU)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


STRONG_SCALING = {5}


def workload_name(cfg, world, strong):
    base = (f"{cfg.name}: TTCLayer fwd+bwd, x[{cfg.B},{cfg.L},{cfg.H},{cfg.in_dim}] per GPU "
            f"as [B, L*H, in] rows, h_dim={cfg.h_dim}, rank={cfg.rank}, T={cfg.T}")
    if cfg.name == "cfg3" and cfg.B == 8 and cfg.L == 4096:
        base += (f"; {cfg.B * world} sequences over {world} GPU(s) (config 5's geometry; at 8 GPUs "
                 "its global batch of 64)")
    elif strong:
        base += f"; config 5's global batch of {cfg.B * world} split over {world} GPU(s)"
    return base


def workload_config(cfg, world, args, chunk, strong=False):
    return {
        "workload": workload_name(cfg, world, strong),
        "B_per_gpu": cfg.B, "L": cfg.L, "H": cfg.H, "in_dim": cfg.in_dim, "out_dim": cfg.out_dim,
        "h_dim": cfg.h_dim, "num_heads": cfg.H, "rank": cfg.rank, "T": cfg.T,
        "rows_per_gpu": cfg.rows, "lqr_problems_per_gpu": cfg.problems,
        "global_batch": cfg.B * world, "activations": cfg.dtype, "solver_state": "f32",
        "parallelism": f"dp{world}" if world > 1 else "single",
        "chunk_rows": chunk, "l2": "rotating input sets larger than L2 (no flush)",
        "solver_impl": args.solver,
    }


# ------------------------------------------------------------------------- main
def main(argv=None):
    args = parse_args(argv)
    cfg = CONFIGS[args.config]
    if args.batch:
        import dataclasses
        cfg = dataclasses.replace(cfg, B=args.batch)
    if args.seq_len:
        import dataclasses
        cfg = dataclasses.replace(cfg, L=args.seq_len)
    if args.workload == "traj":
        if args.warmup < 3:
            raise SystemExit("--warmup must be >= 3")
        return traj_bench(args, cfg)
    if args.impl == "reference":
        return reference_arm(args, cfg)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    # Config 5 is defined at a fixed global batch (64 sequences split over the GPUs):
    # strong scaling.  The other configs keep their per-GPU batch (weak scaling).
    strong = args.config in STRONG_SCALING and not args.batch and not args.seq_len
    if strong:
        import dataclasses
        if cfg.B % world:
            raise SystemExit(f"global batch {cfg.B} of config {args.config} does not split over {world} GPUs")
        cfg = dataclasses.replace(cfg, B=cfg.B // world)
    torch.cuda.set_device(device)
    dtype = torch.bfloat16 if cfg.dtype == "bfloat16" else torch.float32

    from ttc_b200.solver import KernelTimer, set_kernel_timer
    layer = make_layer(cfg, device, dtype, args.solver)
    rows = cfg.L * cfg.H
    chunk = args.chunk_rows or layer.rows_per_call(cfg.rows, dtype, device)

    # Rotating (x, dy) sets on the device, together larger than L2.
    set_bytes = cfg.B * rows * (cfg.in_dim + cfg.out_dim) * (2 if dtype == torch.bfloat16 else 4)
    nsets = max(2, math.ceil(2 * L2_BYTES / set_bytes))
    nsets = min(nsets, 16)
    sets = []
    for s in range(nsets):
        x_np, dy_np = layer_input(cfg, cfg.rows, seed=1000 * rank + s)
        sets.append((torch.from_numpy(x_np).to(device, dtype).view(cfg.B, rows, cfg.in_dim).requires_grad_(True),
                     torch.from_numpy(dy_np).to(device, dtype).view(cfg.B, rows, cfg.out_dim)))

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    reducer = None
    if world > 1:
        from ttc_b200.parallel import OverlappedGradAllReduce
        reducer = OverlappedGradAllReduce(layer)
    for k in range(args.warmup):
        run_step(layer, *sets[k % nsets], cfg.T, chunk, world, reducer)
    torch.cuda.synchronize()

    # ---- device-resident timed region
    timer = KernelTimer()
    phys = gpu_selector(local)
    with ClockSampler(phys) as clocks:
        barrier()
        torch.cuda.synchronize()
        set_kernel_timer(timer)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for k in range(args.steps):
            run_step(layer, *sets[k % nsets], cfg.T, chunk, world, reducer)
        end.record()
        torch.cuda.synchronize()
        set_kernel_timer(None)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    clock_summary = clocks.summary()
    if world > 1:
        import torch.distributed as dist
        every = [None] * world
        dist.all_gather_object(every, clock_summary)
        clock_summary = dict(clock_summary)
        clock_summary["reasons"] = sorted({r for c in every for r in c["reasons"]})
        clock_summary["sm_mhz_per_rank"] = [c["sm_mhz"] for c in every]
    tokens_per_step = cfg.tokens * world
    value = tokens_per_step * args.steps / (ms / 1000.0)
    kern = timer.durations_ms()
    launches = sum(len(v) for v in kern.values())

    # ---- end to end through the public API, host buffers, copies inside the region
    x_host = [torch.from_numpy(layer_input(cfg, cfg.rows, seed=500 + s)[0]).to(dtype).pin_memory()
              for s in range(2)]
    dy_host = [torch.from_numpy(layer_input(cfg, cfg.rows, seed=500 + s)[1]).to(dtype).pin_memory()
               for s in range(2)]
    dx_host = [torch.empty(cfg.rows, cfg.in_dim, dtype=dtype).pin_memory() for _ in range(2)]
    # A data-loader pattern: step k+1's inputs are copied in on a side stream while step k
    # computes, and step k's dx is copied out on it while step k+1 computes.  Every step's
    # copies are inside the timed region (the region ends after the last copy out).
    copy_stream = torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)

    def fetch(k):
        with torch.cuda.stream(copy_stream):
            x = x_host[k % 2].to(device, non_blocking=True).view(cfg.B, rows, cfg.in_dim)
            dy = dy_host[k % 2].to(device, non_blocking=True).view(cfg.B, rows, cfg.out_dim)
            ready = torch.cuda.Event()
            ready.record(copy_stream)
        return x, dy, ready

    def e2e_step(k, inputs):
        x, dy, ready = inputs
        compute.wait_event(ready)
        x.record_stream(compute)
        dy.record_stream(compute)
        x.requires_grad_(True)
        layer.zero_grad(set_to_none=True)
        layer.forward_backward(x, dy, cfg.T, rows=chunk,
                               before_last_backward=reducer.arm if reducer else None)
        if reducer is not None:
            reducer.wait()
        done = torch.cuda.Event()
        done.record(compute)
        gx = x.grad.view(cfg.rows, cfg.in_dim)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(done)
            gx.record_stream(copy_stream)
            dx_host[k % 2].copy_(gx, non_blocking=True)

    # The device-resident loop above is the warm-up of this one (one more step here).  Steps
    # of seconds (configs 3-5) time a quarter of the steps end to end, at least three, so
    # that the whole run stays within a few minutes; the copies are then far below 1 % of a
    # step either way.
    e2e_steps = args.steps if ms / args.steps < 2000.0 else max(3, args.steps // 4)
    e2e_step(0, fetch(0))
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    copy_stream.wait_event(t0)
    nxt = fetch(0)
    for k in range(e2e_steps):
        cur = nxt
        if k + 1 < e2e_steps:
            nxt = fetch(k + 1)
        e2e_step(k, cur)
    compute.wait_stream(copy_stream)
    t1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1))
    es = 2 if dtype == torch.bfloat16 else 4
    h2d = cfg.rows * (cfg.in_dim + cfg.out_dim) * es
    d2h = cfg.rows * cfg.in_dim * es

    if rank == 0:
        fwd_f, bwd_f = solver_flops(cfg)
        fwd_ms = kern.get("ttc_lqr_fwd", [float("nan")])
        # kkt: the backward is one more forward and two rollouts, so the forward launches
        # alternate between the layer's forward and the backward's
        if args.solver == "kkt":
            fwd_ms = fwd_ms[0::2]
        bwd_ms = kern.get("ttc_lqr_bwd", [float("nan")])
        calls_per_step = math.ceil(cfg.rows / chunk)
        probs_per_launch = cfg.problems / calls_per_step
        sm_max = clock_summary.get("sm_max_mhz") or 1965.0
        fp32_peak = SM_COUNT_B200 * FP32_LANES_PER_SM * 2 * sm_max * 1e6 / 1e12
        fwd_tflops = fwd_f * probs_per_launch / (statistics.mean(fwd_ms) / 1e3) / 1e12
        bwd_tflops = bwd_f * probs_per_launch / (statistics.mean(bwd_ms) / 1e3) / 1e12
        traffic = load_traffic(cfg.name, cfg.rows / calls_per_step)
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "f32" if dtype == torch.float32 else "bf16 activations, f32 solver",
            "data": "synthetic (seeded N(0,1) x and dy, reference init distributions)",
            "config": workload_config(cfg, world, args, chunk, strong),
            "roofline": {
                "kernel": "ttc_lqr_fwd (sweep + solve + first step)",
                "bound": "fp32", "achieved": fwd_tflops, "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": fwd_tflops / fp32_peak,
                "peak_source": f"nominal FP32 FMA: 148 SMs x 128 lanes x 2 x {sm_max:.0f} MHz "
                               "(MEASURED_PEAKS.json has no FP32 figure)",
                "flops_per_launch": fwd_f * probs_per_launch,
                "launch_ms": statistics.mean(fwd_ms), "traffic": traffic,
            },
            "kernels": {
                "ttc_lqr_fwd": {"launches": len(fwd_ms), "mean_ms": statistics.mean(fwd_ms),
                                "tflops": fwd_tflops},
                **({"ttc_lqr_bwd": {"launches": len(bwd_ms), "mean_ms": statistics.mean(bwd_ms),
                                    "tflops": bwd_tflops,
                                    "frac_fp32_peak": bwd_tflops / fp32_peak}}
                   if "ttc_lqr_bwd" in kern else {}),
                **{k: {"launches": len(v), "mean_ms": statistics.mean(v)} for k, v in kern.items()
                   if k not in ("ttc_lqr_fwd", "ttc_lqr_bwd")},
            },
            # whole-job rates of the device-resident step (all ranks) and the solver's
            # algorithmic FLOPs (fwd + bwd, solver_flops) per second against the FP32 peak
            "throughput": {
                "rows_per_s": cfg.rows * world * args.steps / (ms / 1000.0),
                "problems_per_s": cfg.problems * world * args.steps / (ms / 1000.0),
                "solver_tflops": (fwd_f + bwd_f) * cfg.problems * world * args.steps / (ms / 1000.0) / 1e12,
                "solver_frac_fp32_peak": (fwd_f + bwd_f) * cfg.problems * args.steps / (ms / 1000.0) / 1e12
                / fp32_peak,
            },
            "clocks": clock_summary,
            "e2e": {"value": tokens_per_step * e2e_steps / (e2e_ms / 1000.0), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "gpu_launches": launches * world,
            "gpu_launches_per_gpu": launches,
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            v, rows_used, dt, kind = cpu_sample(cfg, args.cpu_seconds, threads)
            what = ("the reference's TTCLayer (baseline/_ref, fla l2norm as its formula)" if kind == "reference"
                    else "oracle port of the reference's")
            out["cpu_baseline"] = {
                "value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
                "sample": f"{rows_used} of {cfg.rows} rows ({rows_used / cfg.H:.1f} tokens), "
                          f"{dt:.1f} s: {what} riccati layer fwd + autograd bwd, fp32"}
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------------------------- trajectories
def traj_model(cfg, es):
    """Algorithmic FLOPs and HBM bytes per problem of the rollout kernel (all outputs and the
    affine step-0 term requested)."""
    d = du = cfg.h_dim
    T, nh = cfg.T, cfg.H
    flops = T * 2 * (d * d + 2 * d * du) - 2 * d * d + 2 * d * du + T * 4 * du + 2 * d * d
    out_b = T * du * es + 2 * T * d * 4 + d * 4 + 4
    in_b = (4 * d + 3 * du + 1) * es + d * 4 + d * du * 4 + d * d * es + (d * du + d * d) * es / nh
    return flops, out_b + in_b


def traj_bench(args, cfg):
    """Closed-loop trajectories of every LQR problem of the config's per-GPU batch: one step =
    lqr_trajectory (ttc_lqr_fwd + ttc_lqr_rollout) with actions, states, costates, lambda0, cost
    and an affine step-0 cost, on solver inputs made by the layer's prologue."""
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("--workload traj runs on one GPU")
    from ttc_b200 import lqr_trajectory
    from ttc_b200.solver import KernelTimer, set_kernel_timer
    dtype = torch.bfloat16 if cfg.dtype == "bfloat16" else torch.float32
    es = 2 if dtype == torch.bfloat16 else 4
    flops, nbytes = traj_model(cfg, es)
    rows = args.traj_rows or cfg.rows
    while rows > cfg.H and rows * cfg.H * nbytes > (48 << 30):
        rows //= 2
    problems = rows * cfg.H
    if args.impl == "reference":
        from oracle import ttc_oracle as O
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        layer = O.TTCLayerOracle(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank)
        layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
        sample = min(rows, 256)
        x = torch.from_numpy(layer_input(cfg, sample, seed=3)[0])
        with torch.no_grad():
            ins = layer.solver_inputs(x)
        r0 = torch.randn(ins[0].shape[0], cfg.H, cfg.h_dim)
        vals = []
        for k in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            O.riccati_trajectory(*ins, cfg.T, r_traj=torch.nn.functional.pad(
                r0[:, :, None], (0, 0, 0, cfg.T - 1)))
            if k >= args.warmup:
                vals.append(ins[0].shape[0] * cfg.H / (time.perf_counter() - t0))
        v = statistics.median(vals)
        print(json.dumps({
            "impl": "reference", "metric": "LQR trajectories/s", "value": v, "unit": "trajectories/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "dtype": "f32", "config": {"workload": f"{cfg.name} trajectories, sample of {ins[0].shape[0]} rows"},
            "cpu_baseline": {"value": v, "unit": "trajectories/s", "cores": threads, "kind": "port",
                             "sample": f"{ins[0].shape[0] * cfg.H} problems per step: oracle riccati "
                                       "trajectory + states/costates/cost"}}), flush=True)
        return
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    layer = make_layer(cfg, device, dtype)
    x = torch.from_numpy(layer_input(cfg, rows, seed=3)[0]).to(device, dtype)
    with torch.no_grad():
        ins = layer.solver_inputs(x)
    r0 = torch.randn(rows, cfg.H, cfg.h_dim, device=device).to(dtype)
    want = dict(return_states=True, return_costates=True, return_lambda0=True, return_cost=True)
    for _ in range(args.warmup):
        out = lqr_trajectory(*ins, cfg.T, r0=r0, **want)
        del out
    torch.cuda.synchronize()
    timer = KernelTimer()
    with ClockSampler(gpu_selector(0)) as clocks:
        torch.cuda.synchronize()
        set_kernel_timer(timer)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            out = lqr_trajectory(*ins, cfg.T, r0=r0, **want)
            del out
        end.record()
        torch.cuda.synchronize()
        set_kernel_timer(None)
    ms = start.elapsed_time(end)
    kern = timer.durations_ms()
    roll_ms = statistics.mean(kern["ttc_lqr_rollout"])
    fwd_ms = statistics.mean(kern["ttc_lqr_fwd"])
    peaks = {}
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    clock_summary = clocks.summary()
    sm_max = clock_summary.get("sm_max_mhz") or 1965.0
    fp32_peak = SM_COUNT_B200 * FP32_LANES_PER_SM * 2 * sm_max * 1e6 / 1e12
    gbs = nbytes * problems / (roll_ms / 1e3) / 1e9
    tfl = flops * problems / (roll_ms / 1e3) / 1e12
    print(json.dumps({
        "metric": "LQR trajectories/s", "value": problems * args.steps / (ms / 1e3),
        "unit": "trajectories/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if dtype == torch.float32 else "bf16 inputs, f32 state",
        "data": "synthetic (layer prologue of seeded N(0,1) x; r0 ~ N(0,1))",
        "config": {"workload": f"{cfg.name} trajectories: {rows} rows x {cfg.H} heads, d=du={cfg.h_dim}, "
                               f"T={cfg.T}, actions + states + costates + lambda0 + cost, affine r0",
                   "problems": problems, "l2": "outputs of one step far larger than L2"},
        "roofline": {"kernel": "ttc_lqr_rollout", "bound": "hbm", "achieved": gbs, "peak": hbm,
                     "unit": "GB/s", "frac": gbs / hbm, "bytes_per_problem": nbytes,
                     "launch_ms": roll_ms, "fp32_tflops": tfl, "frac_fp32_peak": tfl / fp32_peak,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        "kernels": {"ttc_lqr_fwd": {"launches": len(kern["ttc_lqr_fwd"]), "mean_ms": fwd_ms},
                    "ttc_lqr_rollout": {"launches": len(kern["ttc_lqr_rollout"]), "mean_ms": roll_ms}},
        "clocks": clock_summary,
        "gpu_launches": sum(len(v) for v in kern.values()),
    }), flush=True)


def load_traffic(workload, rows_per_launch):
    """DRAM bytes per launch of the roofline kernel: the committed ncu capture's bytes per row
    (profiles/traffic.json; the forward's traffic grows with the rows it solves) times the rows
    of one launch."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(p) as f:
            entry = json.load(f).get(workload)
    except (OSError, ValueError):
        return None
    if not entry:
        return None
    return entry["dram_bytes_per_row"] * rows_per_launch


if __name__ == "__main__":
    main()
