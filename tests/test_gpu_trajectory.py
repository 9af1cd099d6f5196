"""GPU parity of the trajectory path (ttc_lqr_fwd or ttc_lqr_fwd_affine + ttc_lqr_rollout
through ``ttc_b200.lqr_trajectory``): closed-loop actions, states, costates, lambda0 and total
cost against the golden vectors of the reference's solve_traj_actions(return_traj=True) and
solve_traj_states (lin_solver_lqr.py:13-212), without an affine cost, with one on step 0 and
with one on every step, and against the oracle's restatement at layer-like sizes."""
import pytest
import torch

from oracle import ttc_oracle as O
from test_oracle_golden import load, solver_args
from test_oracle_traj import OUTS, TRAJ_CASES
from ttc_cases import solver_inputs_synthetic

pytestmark = pytest.mark.gpu

ALL = dict(return_states=True, return_costates=True, return_lambda0=True, return_cost=True)


def _cuda(args, dtype=torch.float32):
    return [a.to("cuda", dtype) for a in args]


@pytest.mark.parametrize("case", TRAJ_CASES)
@pytest.mark.parametrize("tag", ["", "_r0", "_rfull"])
def test_trajectory_matches_reference_golden(case, tag):
    from ttc_b200 import lqr_trajectory
    z = load(case)
    T = int(z["T"])
    r0 = torch.from_numpy(z["r0"]).cuda() if tag == "_r0" else None
    r_traj = torch.from_numpy(z["r_full"]).cuda() if tag == "_rfull" else None
    got = lqr_trajectory(*_cuda(solver_args(z)), T, r0=r0, r_traj=r_traj, **ALL)
    for name, g in zip(OUTS, got):
        ref = torch.from_numpy(z[name + tag])
        assert O.max_rel(g.cpu().double(), ref.double()) < 1e-4, name


def test_first_action_is_the_solver_output():
    from ttc_b200 import cuda_lqr_solve, lqr_trajectory
    z = load("traj_prologue_cfg2")
    args = _cuda(solver_args(z))
    T = int(z["T"])
    u_traj = lqr_trajectory(*args, T)
    u = cuda_lqr_solve(*args, T)
    assert u_traj.shape == (*u.shape[:2], T, u.shape[-1])
    assert O.max_rel(u_traj[:, :, 0], u) < 1e-5


@pytest.mark.parametrize("d,du,nh,N,T", [(16, 16, 16, 96, 64), (32, 32, 32, 6, 128),
                                        (64, 32, 4, 5, 40), (32, 16, 8, 7, 33)])
def test_trajectory_matches_oracle(d, du, nh, N, T):
    """Layer-like sizes against the oracle's fp64 rollout; the affine term included."""
    from ttc_b200 import lqr_trajectory
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(N, nh, d, du, seed=50 + d)]
    g = torch.Generator().manual_seed(d + du)
    r0 = torch.randn(N, nh, du, generator=g, dtype=torch.float64)
    ref = O.fused_trajectory(*host, T, r0=r0)
    got = lqr_trajectory(*_cuda(host), T, r0=r0.cuda(), **ALL)
    for name, a, b in zip(OUTS, got, ref):
        assert O.max_rel(a.cpu().double(), b) < 1e-4, name


@pytest.mark.parametrize("d,du,nh,N,T", [(16, 16, 16, 40, 64), (32, 32, 32, 5, 128),
                                        (64, 32, 4, 3, 40), (32, 16, 8, 7, 33), (16, 16, 3, 4, 1)])
def test_trajectory_with_cost_on_every_step_matches_oracle(d, du, nh, N, T):
    """The per-step affine forward and rollout against the oracle's fp64 restatement (itself
    pinned to the reference's r_traj trajectories), at layer-like sizes."""
    from ttc_b200 import lqr_trajectory
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(N, nh, d, du, seed=70 + d + du)]
    g = torch.Generator().manual_seed(d * du + T)
    r = torch.randn(N, nh, T, du, generator=g, dtype=torch.float64)
    ref = O.fused_trajectory(*host, T, r_traj=r)
    got = lqr_trajectory(*_cuda(host), T, r_traj=r.cuda(), **ALL)
    for name, a, b in zip(OUTS, got, ref):
        assert O.max_rel(a.cpu().double(), b) < 1e-4, name


def test_cost_on_step_zero_only_agrees_with_the_r0_form():
    """r_traj zero after step 0 through ttc_lqr_fwd_affine equals r0 through M: two forwards."""
    from ttc_b200 import lqr_trajectory
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(9, 8, 32, 32, seed=81)]
    args = _cuda(host)
    T = 48
    r0 = torch.randn(9, 8, 32, device="cuda")
    r = torch.zeros(9, 8, T, 32, device="cuda")
    r[:, :, 0] = r0
    a = lqr_trajectory(*args, T, r0=r0, **ALL)
    b = lqr_trajectory(*args, T, r_traj=r, **ALL)
    for name, x, y in zip(OUTS, a, b):
        assert O.max_rel(y.cpu().double(), x.cpu().double()) < 1e-5, name


def test_row_chunks_give_the_same_trajectory():
    """A save budget of a few rows splits the launches into row chunks: same bits."""
    from ttc_b200 import lqr_trajectory
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(11, 4, 16, 16, seed=60)]
    args = _cuda(host)
    r0 = torch.randn(11, 4, 16, device="cuda")
    whole = lqr_trajectory(*args, 24, r0=r0, **ALL)
    chunked = lqr_trajectory(*args, 24, r0=r0, save_budget=3 * 4 * 16 * 16 * 4, **ALL)
    for a, b in zip(whole, chunked):
        assert torch.equal(a, b)


def test_affine_lambda0_is_the_backward_h0_gradient():
    """h0 = 0, r0 = du: lambda0 of the trajectory is the kkt second problem's lambda0,
    i.e. the h0 gradient of the solve (torch_lqr.py:41-47,63) -- two kernels, one answer."""
    from ttc_b200 import cuda_lqr_solve, lqr_trajectory
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(64, 16, 16, 16, seed=61)]
    args = [a.cuda().float().requires_grad_(True) for a in host]
    T = 64
    u = cuda_lqr_solve(*args, T)
    dy = torch.randn_like(u)
    (u * dy).sum().backward()
    plain = [a.detach() for a in args]
    lam0 = lqr_trajectory(*plain[:8], torch.zeros_like(plain[8]), T, r0=dy,
                          return_lambda0=True)[1]
    assert O.max_rel(lam0, args[8].grad) < 1e-4


def test_bf16_trajectory_matches_oracle():
    """bf16 inputs: fp32 state inside, u in bf16; against the oracle on the bf16-rounded
    inputs (2e-2, the bf16 bar of the solver)."""
    from ttc_b200 import lqr_trajectory
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(8, 8, 32, 32, seed=62)]
    rounded = [a.to(torch.bfloat16).double() for a in host]
    ref = O.fused_trajectory(*rounded, 32)
    got = lqr_trajectory(*_cuda(host, torch.bfloat16), 32, return_states=True)
    assert got[0].dtype == torch.bfloat16 and got[1].dtype == torch.float32
    assert O.max_rel(got[0].cpu().double(), ref[0]) < 2e-2
    assert O.max_rel(got[1].cpu().double(), ref[1]) < 2e-2


def test_trajectory_errors():
    from ttc_b200 import lqr_trajectory
    host = [torch.from_numpy(a).float() for a in solver_inputs_synthetic(2, 2, 16, 16, seed=63)]
    args = _cuda(host)
    with pytest.raises(AssertionError, match="r_traj"):
        lqr_trajectory(*args, 8, r0=torch.zeros(2, 2, 8, 16, device="cuda"))  # every step: r_traj
    with pytest.raises(AssertionError, match="r_traj must be"):
        lqr_trajectory(*args, 8, r_traj=torch.zeros(2, 2, 7, 16, device="cuda"))
    with pytest.raises(ValueError, match="not both"):
        lqr_trajectory(*args, 8, r0=torch.zeros(2, 2, 16, device="cuda"),
                       r_traj=torch.zeros(2, 2, 8, 16, device="cuda"))
    with pytest.raises(ValueError):
        lqr_trajectory(*host, 8)  # CPU tensors: there is no CPU path
    bad = list(args)
    bad[8] = bad[8].clone()
    bad[8][0, 0, 0] = float("nan")
    with pytest.raises(RuntimeError, match="Non-finite"):
        lqr_trajectory(*bad, 8)
