"""Pin the trajectory oracle to the reference: riccati_trajectory (the reference's
solve_traj_actions(return_traj=True) + solve_traj_states semantics) and fused_trajectory (the
forward-in-time rollout the CUDA path runs) against golden vectors made by running the
reference's lin_solver_lqr (tests/golden/make_golden.py traj_case)."""
import numpy as np
import pytest
import torch

from oracle import ttc_oracle as O
from test_oracle_golden import load, solver_args

TRAJ_CASES = ["traj_bench_d16", "traj_prologue_cfg2", "traj_synth_d32_du16", "traj_T1"]
OUTS = ["u_traj", "states", "costates", "lambda0", "cost"]


def _golden(z, tag):
    return [torch.from_numpy(z[k + tag]).double() for k in OUTS]


@pytest.mark.parametrize("case", TRAJ_CASES)
@pytest.mark.parametrize("tag", ["", "_r0", "_rfull"])
def test_riccati_trajectory_matches_reference(case, tag):
    z = load(case)
    T = int(z["T"])
    r = None
    if tag == "_r0":
        r = torch.zeros(*z["r0"].shape[:2], T, z["r0"].shape[-1])
        r[:, :, 0] = torch.from_numpy(z["r0"])
    elif tag == "_rfull":
        r = torch.from_numpy(z["r_full"])
    got = O.riccati_trajectory(*solver_args(z), T, r_traj=r)
    for name, g, ref in zip(OUTS, got, _golden(z, tag)):
        assert O.max_rel(g.double(), ref) < 1e-4, name


@pytest.mark.parametrize("case", TRAJ_CASES)
@pytest.mark.parametrize("tag", ["", "_r0"])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_fused_trajectory_matches_reference(case, tag, dtype):
    """The forward-in-time rollout from lambda0 (+ M r0) reproduces the reference's
    Riccati trajectories: actions, states, costates, lambda0 and total cost."""
    z = load(case)
    T = int(z["T"])
    r0 = torch.from_numpy(z["r0"]).to(dtype) if tag else None
    got = O.fused_trajectory(*solver_args(z, dtype), T, r0=r0)
    for name, g, ref in zip(OUTS, got, _golden(z, tag)):
        assert O.max_rel(g.double(), ref) < 1e-4, name


@pytest.mark.parametrize("case", TRAJ_CASES)
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_fused_trajectory_with_cost_on_every_step_matches_reference(case, dtype):
    """The per-step affine sweep (the offset c of each row, lambda0 = Y1^-1 (Y2 h0 + c)) and
    the rollout with -R_inv r_k on every step reproduce the reference's Riccati trajectories
    with r_traj on every step."""
    z = load(case)
    T = int(z["T"])
    r = torch.from_numpy(z["r_full"]).to(dtype)
    got = O.fused_trajectory(*solver_args(z, dtype), T, r_traj=r)
    for name, g, ref in zip(OUTS, got, _golden(z, "_rfull")):
        assert O.max_rel(g.double(), ref) < 1e-4, name


def test_fused_forward_per_step_affine_reduces_to_step0_form():
    """With r_traj zero after step 0 the per-step offset c is Y3 r0 (IS_AFFINE)."""
    z = load("traj_bench_d16")
    args = solver_args(z, torch.float64)
    T = int(z["T"])
    r0 = torch.from_numpy(z["r0"]).double()
    r = torch.zeros(*r0.shape[:2], T, r0.shape[-1], dtype=torch.float64)
    r[:, :, 0] = r0
    u_a, lam_a = O.fused_forward(*args, T, r_traj=r)[:2]
    _, lam, Y1, _, Y3, _ = O.fused_forward(*args, T)
    lam_b = lam + torch.linalg.solve(Y1, Y3 @ r0[..., None])[..., 0]
    assert O.max_rel(lam_a, lam_b) < 1e-10


def test_fused_trajectory_first_action_is_the_solve():
    """u_traj[..., 0, :] is the solver output u of the same inputs."""
    z = load("traj_bench_d16")
    args = solver_args(z, torch.float64)
    T = int(z["T"])
    u_traj = O.fused_trajectory(*args, T)[0]
    u = O.fused_forward(*args, T)[0]
    assert torch.equal(u_traj[:, :, 0], u)


def test_affine_step0_equals_kkt_second_problem():
    """With h0 = 0 and r0 = du the trajectory is the kkt backward's second LQR
    (torch_lqr.py:41-47): its lambda0 is the h0 gradient the kkt solver returns."""
    z = load("solver_bench_d16")
    args = solver_args(z, torch.float64)
    T = int(z["T"])
    dy = torch.from_numpy(z["dy"]).double()
    zero_h0 = torch.zeros_like(args[8])
    lam0 = O.fused_trajectory(*args[:8], zero_h0, T, r0=dy)[3]
    assert O.max_rel(lam0, torch.from_numpy(z["g_h0"]).double()) < 1e-3
