"""Generate the golden vectors that pin the CPU oracle to the reference itself.

Runs the reference package (VITA-Group/TTC-Net ``ttc/``) on the CPU -- its
``riccati`` and ``kkt`` solvers and its ``TTCLayer`` -- and stores inputs and
outputs as compressed .npz fixtures beside this script.  The reference must be
importable (set TTC_REFERENCE_ROOT to its checkout); it is NOT needed
to run the tests, which only read the fixtures.

fla's Triton ``l2norm`` wrapper does not run on CPU tensors, so
``ttc.layers.ttc_layer.l2norm`` is replaced by the same formula
(x / sqrt(sum x^2 + 1e-6), fp32 compute, cast back -- fla/modules/l2norm.py:42).
The Triton ``fused`` solver needs CUDA and is not run here.

Usage:  TTC_REFERENCE_ROOT=<checkout> python tests/golden/make_golden.py        (all fixtures)
        TTC_REFERENCE_ROOT=<checkout> python tests/golden/make_golden.py traj   (trajectory fixtures only)
        TTC_REFERENCE_ROOT=<checkout> python tests/golden/make_golden.py cfg5   (config-5 and bf16-gradient fixtures only)
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))          # tests/ for ttc_cases
from ttc_cases import CONFIGS, SOLVER_ARG_NAMES, layer_input, layer_weights, solver_inputs_synthetic  # noqa: E402

REF = os.environ.get("TTC_REFERENCE_ROOT")
if not REF:
    raise SystemExit("set TTC_REFERENCE_ROOT to the reference (VITA-Group/TTC-Net) checkout")
sys.path.insert(0, REF)
os.environ.setdefault("TRITON_NO_AUTOTUNE", "1")
import ttc.layers.ttc_layer as ref_layer_mod  # noqa: E402
from ttc.solvers.lin_solver_lqr import solve_traj_actions, solve_traj_states  # noqa: E402
from ttc.solvers.torch_lqr import _generate_parameters, direct_lqr_solve, kkt_lqr_solve  # noqa: E402


def _l2norm_cpu(x, eps=1e-6):
    xf = x.float()
    return (xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


ref_layer_mod.l2norm = _l2norm_cpu
RefTTCLayer = ref_layer_mod.TTCLayer

GRAD_NAMES = ["g_" + n for n in SOLVER_ARG_NAMES]
MAX_FIXTURE_FLOATS = 32768


def _np(t):
    return t.detach().to(torch.float32).cpu().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()


def solver_case(name, args, T, seed_dy, dtype=torch.float32, with_kkt=True):
    """riccati u and kkt u + 9 gradients for one set of solver inputs."""
    t0 = time.time()
    args = [torch.as_tensor(a).to(dtype) for a in args]
    out = {n: _np(a) for n, a in zip(SOLVER_ARG_NAMES, args)}
    out["T"] = np.array(T)
    with torch.no_grad():
        out["u_riccati"] = _np(direct_lqr_solve(*args, T))
    if with_kkt:
        leaves = [a.clone().requires_grad_(True) for a in args]
        u = kkt_lqr_solve(*leaves, T)
        g = torch.from_numpy(np.random.default_rng(seed_dy).standard_normal(u.shape)).to(dtype)
        (u * g).sum().backward()
        out["dy"] = _np(g)
        out["u_kkt"] = _np(u)
        for gn, leaf in zip(GRAD_NAMES, leaves):
            out[gn] = _np(leaf.grad)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)


def capture_prologue(cfg, rows, heads=None):
    """Solver inputs produced by the reference TTCLayer prologue (ttc_layer.py:104-135)."""
    layer = RefTTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                        solver_impl="riccati")
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    x, _ = layer_input(cfg, rows)
    box = {}

    def grab(*a):
        box["a"] = a
        return torch.zeros_like(a[0])

    layer.solver = grab
    with torch.no_grad():
        layer(torch.from_numpy(x)[None], T=cfg.T)
    args = [a.detach().clone() for a in box["a"][:9]]
    if heads is not None:
        per_head = [0, 3, 4, 5, 6, 7, 8]        # B (1) and Q (2) are per row
        for i in per_head:
            args[i] = args[i][:, :heads].contiguous()
    return args


def layer_case(name, cfg, rows, dtype=torch.float32, solver="kkt", backward=True):
    """Reference TTCLayer forward (and kkt backward) on `rows` rows of config `cfg`."""
    t0 = time.time()
    layer = RefTTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                        solver_impl=solver)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    layer = layer.to(dtype)
    x_np, dy_np = layer_input(cfg, rows)
    x = torch.from_numpy(x_np).to(dtype)[None].requires_grad_(backward)
    y = layer(x, T=cfg.T)
    out = {"x": x_np, "y": _np(y[0]), "T": np.array(cfg.T), "rows": np.array(rows),
           "cfg": np.array(int(cfg.name[3:]))}
    if backward:
        dy = torch.from_numpy(dy_np).to(dtype)[None]
        (y * dy).sum().backward()
        out["dy"] = dy_np
        out["g_x"] = _np(x.grad[0])
        for pn, p in layer.named_parameters():
            g = _np(p.grad)
            # Large weight gradients keep every `stride`-th row so fixtures stay small;
            # the tests compare the same rows.
            stride = max(1, -(-g.size // MAX_FIXTURE_FLOATS))
            out["g_" + pn] = g[::stride]
            out["stride_" + pn] = np.array(stride)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)


def traj_case(name, args, T, seed_r):
    """Closed-loop trajectories from the reference's lin_solver_lqr on the time-varying
    system of torch_lqr._generate_parameters: without an affine term, with an affine action
    cost r0 on step 0 only (the kkt backward's form), and with an affine cost on every step."""
    t0 = time.time()
    args = [torch.as_tensor(a).to(torch.float32) for a in args]
    out = {n: _np(a) for n, a in zip(SOLVER_ARG_NAMES, args)}
    out["T"] = np.array(T)
    N, nh, d = args[0].shape
    du = args[1].shape[-1]
    A_t, B_t, Q_t, R_t = _generate_parameters(*args[:8], T)
    A_t, B_t = A_t.reshape(-1, T, d), B_t.reshape(-1, T, d, du)
    Q_t, R_t = Q_t.reshape(-1, T, d, d), R_t.reshape(-1, T, du)
    h0 = args[8].reshape(-1, d)
    rng = np.random.default_rng(seed_r)
    r0 = torch.from_numpy(rng.standard_normal((N, nh, du))).float()
    r_full = torch.from_numpy(rng.standard_normal((N, nh, T, du))).float()
    r_step0 = torch.zeros(N * nh, T, du)
    r_step0[:, 0] = r0.reshape(-1, du)
    out["r0"] = _np(r0)
    out["r_full"] = _np(r_full)
    with torch.no_grad():
        for tag, r in (("", None), ("_r0", r_step0), ("_rfull", r_full.reshape(-1, T, du))):
            u = solve_traj_actions(A_t, B_t, Q_t, R_t, h0, r_traj=r, return_traj=True)
            cost, hs, lam, lam0 = solve_traj_states(u, A_t, B_t, Q_t, R_t, h0, r_traj=r,
                                                    return_states=True, return_costates=True,
                                                    return_lambda0=True)
            out["u_traj" + tag] = _np(u.reshape(N, nh, T, du))
            out["states" + tag] = _np(hs.reshape(N, nh, T, d))
            out["costates" + tag] = _np(lam.reshape(N, nh, T, d))
            out["lambda0" + tag] = _np(lam0.reshape(N, nh, d))
            out["cost" + tag] = _np(cost.reshape(N, nh))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)


def traj_cases():
    """Trajectory fixtures (solve_traj_actions(return_traj=True) + solve_traj_states)."""
    from ttc.solvers.bench_lqr_solvers import generate_inputs
    torch.manual_seed(0)
    A, B, Q, R, Qf, lgA, lgB, lgQ, h0 = generate_inputs(2, 3, 16, torch.device("cpu"),
                                                        torch.float32, 64, False)
    Q = (Q + Q.transpose(-1, -2)) / 2
    Qf = (Qf + Qf.transpose(-1, -2)) / 2
    traj_case("traj_bench_d16", [A, B, Q, R, Qf, lgA, lgB, lgQ, h0], 64, seed_r=40)
    traj_case("traj_prologue_cfg2", capture_prologue(CONFIGS[2], 2, heads=4), 64, seed_r=41)
    traj_case("traj_synth_d32_du16", solver_inputs_synthetic(2, 2, 32, 16, seed=6), 32, seed_r=42)
    traj_case("traj_T1", solver_inputs_synthetic(2, 2, 16, 16, seed=7), 1, seed_r=43)


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    # 1. The reference's own correctness-check case (bench_lqr_solvers.py:173-207):
    #    bs=4, nh=4, d=16, T=64 from its generate_inputs with torch seed 0, Q/Q_f
    #    symmetrised before the solve (:125,127).
    from ttc.solvers.bench_lqr_solvers import generate_inputs
    torch.manual_seed(0)
    A, B, Q, R, Qf, lgA, lgB, lgQ, h0 = generate_inputs(4, 4, 16, torch.device("cpu"),
                                                        torch.float32, 64, False)
    Q = (Q + Q.transpose(-1, -2)) / 2
    Qf = (Qf + Qf.transpose(-1, -2)) / 2
    solver_case("solver_bench_d16", [A, B, Q, R, Qf, lgA, lgB, lgQ, h0], 64, seed_dy=10)

    # 2. Synthetic solver inputs at other geometries and edge horizons.
    solver_case("solver_synth_d32", solver_inputs_synthetic(2, 4, 32, 32, seed=1), 32, seed_dy=11)
    solver_case("solver_synth_d64", solver_inputs_synthetic(1, 2, 64, 64, seed=2), 48, seed_dy=12)
    solver_case("solver_T1", solver_inputs_synthetic(3, 2, 16, 16, seed=3), 1, seed_dy=13)
    solver_case("solver_T2", solver_inputs_synthetic(3, 2, 16, 16, seed=4), 2, seed_dy=14)
    # State growth (~3e5 over T=64) that trips the 1e3 renormalisation of the symplectic
    # sweep while staying well conditioned in fp32: gamma_A = e^-0.02 keeps A_t near
    # 1 + A_diag.  (At ~1e10 growth and beyond, the reference's symplectic fp32 sweep
    # itself departs from riccati, so such inputs pin nothing.)
    g = solver_inputs_synthetic(2, 3, 16, 16, seed=5)
    g[5] = np.full_like(g[5], -0.02)
    g[0] = g[0] * 0.5
    solver_case("solver_growth", g, 64, seed_dy=15)

    # 3. Inputs captured from the reference layer prologue at each config geometry.
    solver_case("prologue_cfg1", capture_prologue(CONFIGS[1], 4), 64, seed_dy=21)
    solver_case("prologue_cfg2", capture_prologue(CONFIGS[2], 2), 64, seed_dy=22)
    solver_case("prologue_cfg3", capture_prologue(CONFIGS[3], 1, heads=8), 128, seed_dy=23)
    solver_case("prologue_cfg4", capture_prologue(CONFIGS[4], 1, heads=4), 512, seed_dy=24)
    solver_case("prologue_cfg3_bf16", capture_prologue(CONFIGS[3], 1, heads=8), 128,
                seed_dy=25, dtype=torch.bfloat16, with_kkt=False)

    # 4. Whole-layer cases: y from the reference TTCLayer, gradients from its kkt
    #    solver (same symmetric Q convention as the fused backward).
    layer_case("layer_cfg1", CONFIGS[1], 16, solver="riccati", backward=False)
    layer_case("layer_cfg2", CONFIGS[2], 32)
    layer_case("layer_cfg3", CONFIGS[3], 4)
    layer_case("layer_cfg4", CONFIGS[4], 1)
    layer_case("layer_cfg3_bf16", CONFIGS[3], 4, dtype=torch.bfloat16, solver="riccati",
               backward=False)
    # 5. Config 5 (seed 4; config 3's geometry): fp32 y and kkt gradients, and the bf16
    #    cases below.
    layer_case("layer_cfg5", CONFIGS[5], 4)
    bf16_layer_cases()


def bf16_layer_cases():
    """bf16-activation layers (configs 3 and 5): the recommended oracle, fp32 y and kkt
    gradients on the bf16-rounded x, dy and weights, next to the reference's own bf16 forward
    (riccati; the reference's kkt backward does not run in bf16: its Riccati solve mixes
    float and bfloat16 operands, lin_solver_lqr.py:6)."""
    for cid in (3, 5):
        cfg = CONFIGS[cid]
        t0 = time.time()
        x_np, dy_np = layer_input(cfg, 4)
        w = {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in layer_weights(cfg).items()}
        xb = torch.from_numpy(x_np).to(torch.bfloat16)
        dyb = torch.from_numpy(dy_np).to(torch.bfloat16)
        out = {"x": x_np, "dy": dy_np, "T": np.array(cfg.T), "rows": np.array(4), "cfg": np.array(cid)}
        layer = RefTTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                            solver_impl="kkt")
        layer.load_state_dict({k: v.float() for k, v in w.items()})
        x = xb.float()[None].requires_grad_(True)
        y = layer(x, T=cfg.T)
        (y * dyb.float()[None]).sum().backward()
        out["y"] = _np(y[0])
        out["g_x"] = _np(x.grad[0])
        for pn, p in layer.named_parameters():
            g = _np(p.grad)
            stride = max(1, -(-g.size // MAX_FIXTURE_FLOATS))
            out["g_" + pn] = g[::stride]
            out["stride_" + pn] = np.array(stride)
        ref16 = RefTTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                            solver_impl="riccati")
        ref16.load_state_dict({k: v.float() for k, v in w.items()})
        ref16 = ref16.to(torch.bfloat16)
        with torch.no_grad():
            out["y_refbf16"] = _np(ref16(xb[None], T=cfg.T)[0])
        np.savez_compressed(os.path.join(HERE, f"layer_cfg{cid}_bf16grad.npz"), **out)
        print(f"layer_cfg{cid}_bf16grad: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    if sys.argv[1:] == ["traj"]:
        torch.set_num_threads(os.cpu_count() or 1)
        traj_cases()
    elif sys.argv[1:] == ["cfg5"]:
        torch.set_num_threads(os.cpu_count() or 1)
        layer_case("layer_cfg5", CONFIGS[5], 4)
        bf16_layer_cases()
    else:
        main()
        traj_cases()
