"""Golden vectors and timings from the reference's own GPU solver (the Triton ``fused`` path).

The reference's default solver, ``fused_lqr_solve`` (ttc/solvers/fused_lqr.py:255-304, Triton
kernels in ttc/solvers/symplectic_iter.py), needs CUDA and Triton, so this script runs on a
B200 box, not in the build container.  The reference package must be importable there: set
TTC_REFERENCE_ROOT to a directory holding the ``ttc`` package (an unmodified install of the
reference, e.g. ``baseline/_ref`` made by ``pip install --target``); fla and triton come from
the image.  The tests only read the fixtures this writes.

    TTC_REFERENCE_ROOT=baseline/_ref python tests/golden/make_fused_golden.py golden OUT_DIR
    TTC_REFERENCE_ROOT=baseline/_ref python tests/golden/make_fused_golden.py time OUT_JSON

``golden``: for every solver fixture of make_golden.py (its inputs and upstream gradient), the
fused solver's u and nine gradients (fp32) -> ``fused_<case>.npz``; solver inputs captured
from the reference layer prologue at the geometry of configs 3 and 5 (2 rows, all 32 heads)
with the fused u and gradients -> ``fused_capture_cfg{3,5}.npz``; and whole-layer cases,
``TTCLayer(solver_impl="fused")`` on the GPU, y and the gradients of x and of every parameter
-> ``fused_layer_cfg{3,5}.npz`` (fp32) and ``fused_layer_cfg5_bf16.npz`` (bf16 activations).
Triton autotuning is off (TRITON_NO_AUTOTUNE=1, the reference's switch) so the fixtures come
from one fixed kernel configuration.

``time``: forward + backward of the fused solver against ``ttc_b200``'s CUDA solver on the same
inputs (the reference benchmark's generator, bench_lqr_solvers.py:71-101, as its
run_correctness_check does, :173-207) at config 2 (all 65 536 rows, fp32) and at config-3
geometry (32 768 rows, bf16), CUDA events, Triton autotuning on.
"""
from __future__ import annotations

import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for _p in (os.path.dirname(HERE), os.path.join(REPO, "ttc-net_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)
from ttc_cases import CONFIGS, SOLVER_ARG_NAMES, layer_input, layer_weights  # noqa: E402

# every solver fixture of make_golden.py except prologue_cfg3 (8 of its 32 heads), which the
# capture below covers with all 32 heads
SOLVER_CASES = ["solver_bench_d16", "solver_synth_d32", "solver_synth_d64", "solver_T1",
                "solver_T2", "solver_growth", "prologue_cfg1", "prologue_cfg2", "prologue_cfg4"]
GRAD_NAMES = ["g_" + n for n in SOLVER_ARG_NAMES]
MAX_FIXTURE_FLOATS = 32768


def _reference():
    root = os.environ.get("TTC_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set TTC_REFERENCE_ROOT to a directory holding the reference's ttc package")
    sys.path.insert(0, os.path.abspath(root))
    import ttc.layers.ttc_layer as layer_mod
    from ttc.solvers.fused_lqr import fused_lqr_solve
    return layer_mod.TTCLayer, fused_lqr_solve


def _np(t):
    return t.detach().float().cpu().numpy()


def fused_case(fused, args, T, dy):
    """u and the nine gradients of the reference's fused solver for one set of inputs."""
    leaves = [a.detach().clone().cuda().requires_grad_(True) for a in args]
    u = fused(*leaves, T)
    (u * dy.to(u.dtype)).sum().backward()
    torch.cuda.synchronize()
    out = {n: _np(a) for n, a in zip(SOLVER_ARG_NAMES, leaves)}
    out.update({"T": np.array(T), "dy": _np(dy), "u_fused": _np(u)})
    out.update({gn: _np(leaf.grad) for gn, leaf in zip(GRAD_NAMES, leaves)})
    return out


def capture_prologue(RefLayer, cfg, rows):
    """Solver inputs made by the reference layer prologue (ttc_layer.py:104-135) on the GPU."""
    layer = RefLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                     solver_impl="riccati").cuda()
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    x, _ = layer_input(cfg, rows)
    box = {}

    def grab(*a):
        box["a"] = a
        return torch.zeros_like(a[0])

    layer.solver = grab
    with torch.no_grad():
        layer(torch.from_numpy(x).cuda()[None], T=cfg.T)
    return [a.detach().float().contiguous() for a in box["a"][:9]]


def layer_case(RefLayer, cfg, rows, dtype):
    """TTCLayer(solver_impl="fused") forward + backward on `rows` rows of config `cfg`."""
    layer = RefLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                     solver_impl="fused")
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    layer = layer.to("cuda", dtype)
    x_np, dy_np = layer_input(cfg, rows)
    x = torch.from_numpy(x_np).to("cuda", dtype)[None].requires_grad_(True)
    y = layer(x, T=cfg.T)
    (y * torch.from_numpy(dy_np).to("cuda", dtype)[None]).sum().backward()
    torch.cuda.synchronize()
    out = {"x": x_np, "dy": dy_np, "y": _np(y[0]), "g_x": _np(x.grad[0]), "T": np.array(cfg.T),
           "rows": np.array(rows), "cfg": np.array(int(cfg.name[3:]))}
    for pn, p in layer.named_parameters():
        g = _np(p.grad)
        stride = max(1, -(-g.size // MAX_FIXTURE_FLOATS))
        out["g_" + pn] = g[::stride]
        out["stride_" + pn] = np.array(stride)
    return out


def golden(out_dir):
    os.environ.setdefault("TRITON_NO_AUTOTUNE", "1")
    RefLayer, fused = _reference()
    os.makedirs(out_dir, exist_ok=True)

    def save(name, out):
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **out)
        print(f"{name}: written", flush=True)

    for case in SOLVER_CASES:
        z = np.load(os.path.join(HERE, case + ".npz"))
        args = [torch.from_numpy(z[n]).float().cuda() for n in SOLVER_ARG_NAMES]
        T = int(z["T"])
        dy = torch.from_numpy(z["dy"]).float().cuda()
        save("fused_" + case, fused_case(fused, args, T, dy))
    for cid, seed_dy in ((3, 33), (5, 35)):
        cfg = CONFIGS[cid]
        args = capture_prologue(RefLayer, cfg, 2)
        g = np.random.default_rng(seed_dy).standard_normal(tuple(args[3].shape))
        dy = torch.from_numpy(g).float().cuda()
        save(f"fused_capture_cfg{cid}", fused_case(fused, args, cfg.T, dy))
    save("fused_layer_cfg3", layer_case(RefLayer, CONFIGS[3], 8, torch.float32))
    save("fused_layer_cfg5", layer_case(RefLayer, CONFIGS[5], 8, torch.float32))
    save("fused_layer_cfg5_bf16", layer_case(RefLayer, CONFIGS[5], 8, torch.bfloat16))


def _time_fwd_bwd(solve, args, T, dy, warmup=2, steps=5):
    for _ in range(warmup):
        leaves = [a.detach().requires_grad_(True) for a in args]
        (solve(*leaves, T) * dy).sum().backward()
    torch.cuda.synchronize()
    leaves_all = [[a.detach().requires_grad_(True) for a in args] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for leaves in leaves_all:
        (solve(*leaves, T) * dy).sum().backward()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def timing(out_json):
    _, fused = _reference()
    from ttc.solvers.bench_lqr_solvers import generate_inputs
    from ttc_b200 import cuda_lqr_solve
    results = []
    for name, N, nh, d, T, dtype in (("cfg2 (all 65 536 rows)", 65536, 16, 16, 64, torch.float32),
                                     ("cfg3 geometry (32 768 rows)", 32768, 32, 32, 128, torch.bfloat16)):
        torch.manual_seed(0)
        args = list(generate_inputs(N, nh, d, torch.device("cuda"), dtype, T, False))
        args[2] = ((args[2] + args[2].transpose(-1, -2)) / 2).contiguous()
        args[4] = ((args[4] + args[4].transpose(-1, -2)) / 2).contiguous()
        dy = torch.randn(N, nh, d, device="cuda").to(dtype)
        t0 = time.time()
        ms_fused = _time_fwd_bwd(fused, args, T, dy)
        tune_s = time.time() - t0
        ms_cuda = _time_fwd_bwd(cuda_lqr_solve, args, T, dy)
        fwd = T * 4 * d**3 + (T - 1) * 2 * d**3 + (8 / 3) * d**3 + 4 * d * d + 4 * d * d
        bwd = T * 20 * d * d + 4 * d * d
        flops = (fwd + bwd) * N * nh
        r = {"workload": name, "problems": N * nh, "d": d, "T": T, "dtype": str(dtype),
             "fused_triton_ms": ms_fused, "cuda_ms": ms_cuda, "speedup": ms_fused / ms_cuda,
             "fused_tflops": flops / ms_fused / 1e9, "cuda_tflops": flops / ms_cuda / 1e9,
             "fused_first_calls_s": tune_s}
        print(json.dumps(r), flush=True)
        results.append(r)
        del args, dy
        torch.cuda.empty_cache()
    meta = {"gpu": torch.cuda.get_device_name(0), "torch": torch.__version__}
    try:
        import triton
        meta["triton"] = triton.__version__
        import fla
        meta["fla"] = getattr(fla, "__version__", "?")
    except ImportError:
        pass
    with open(out_json, "w") as f:
        json.dump({"meta": meta, "results": results}, f, indent=1)


if __name__ == "__main__":
    if len(sys.argv) != 3 or sys.argv[1] not in ("golden", "time"):
        raise SystemExit(__doc__)
    torch.backends.cuda.matmul.allow_tf32 = False
    if sys.argv[1] == "golden":
        golden(sys.argv[2])
    else:
        timing(sys.argv[2])
