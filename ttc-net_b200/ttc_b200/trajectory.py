"""Closed-loop trajectories of the LQR solve on the GPU.

The reference computes trajectories with its Riccati solver
(``solve_traj_actions(..., r_traj, return_traj=True)``, ttc/solvers/lin_solver_lqr.py:113-212)
and rolls out states, costates and the total cost with ``solve_traj_states`` (:13-110); its
kkt backward runs both, once with an affine action cost ``r_0`` on step 0
(ttc/solvers/torch_lqr.py:41-47), and its symplectic sweep carries the same affine term as
``IS_AFFINE`` (y3 = Y3 r, ttc/solvers/symplectic_iter.py:211-238).  ``lqr_trajectory`` gives
those outputs for the layer's solver inputs in two launches per row chunk: ``ttc_lqr_fwd``
(sweep + solve: lambda0 = P h0 and, with r0, M = Y1^-1 Y3) and ``ttc_lqr_rollout`` (the
forward-in-time state / costate recursion of the reference's adjoint primal).

Affine terms: ``r0`` [N, nh, du] on step 0 only -- the form both reference users take -- or
``r_traj`` [N, nh, T, du], a cost r_t^T u_t on every step (the reference's r_traj).  For the
latter the forward is ``ttc_lqr_fwd_affine``: the sweep carries the offset c of each row's
constraint Y1 lambda = Y2 h + c, lambda0 solves Y1 lambda0 = Y2 h0 + c, and the rollout
subtracts R_inv r_t from every step's action.

The outputs are detached: no autograd graph is recorded through this call.
"""
from __future__ import annotations

import torch

from . import _lib
from .solver import (SAVE_BUDGET_BYTES, _DTYPES, _check_shapes, _flags, _launch, _prepare, _ptr,
                     check_fwd_status)

TRAJ_NONFINITE_MSG = "Non-finite value in the LQR trajectory rollout."


def lqr_trajectory(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                   r0=None, return_states: bool = False, return_costates: bool = False,
                   return_lambda0: bool = False, return_cost: bool = False,
                   inv_guard: bool = False, save_budget: int | None = None, r_traj=None):
    """Closed-loop action trajectory u_t, t = 0..T-1, of every problem: [N, nh, T, du] in the
    inputs' dtype (u_traj[:, :, 0] is the solver's u).  Inputs as the layer's solver
    (ttc_layer.py:137); ``r0`` [N, nh, du] adds the affine action cost r0^T u_0, ``r_traj``
    [N, nh, T, du] the cost r_t^T u_t on every step (at most one of the two).

    With any ``return_*`` flag, returns a tuple (u_traj, then in this order the ones asked
    for): states [N, nh, T, d] = h_1..h_T, costates [N, nh, T, d] = lambda_1..lambda_T,
    lambda0 [N, nh, d], cost [N, nh] (sum_t 0.5 h_{t+1}^T Q_t h_{t+1} + 0.5 u_t^T R_t u_t
    + r_t^T u_t with Q_{T-1} = Q_f, R_t = 1 / R_inv) -- float32, as solve_traj_states.
    Row chunks keep the forward's M (needed for r0) within ``save_budget`` bytes."""
    T = int(T)
    N, nh, d, du = _check_shapes(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B,
                                 log_gamma_Q, h0, T)
    dtype = Q.dtype
    if dtype not in _DTYPES:
        raise TypeError(f"ttc_b200 trajectory supports float32 and bfloat16, got {dtype}")
    if r0 is not None and r_traj is not None:
        raise ValueError("pass either r0 (step 0) or r_traj (every step), not both")
    if r0 is not None and tuple(r0.shape) != (N, nh, du):
        hint = "; an affine cost on every step goes in r_traj" if r0.dim() == 4 else ""
        raise AssertionError(f"r0 must be [{N},{nh},{du}], got {tuple(r0.shape)}{hint}")
    if r_traj is not None and tuple(r_traj.shape) != (N, nh, T, du):
        raise AssertionError(f"r_traj must be [{N},{nh},{T},{du}], got {tuple(r_traj.shape)}")
    dev = Q.device
    budget = SAVE_BUDGET_BYTES if save_budget is None else int(save_budget)
    with torch.no_grad():
        A, Bm, Qm, R, Qf, lA, lB, lQ, H0 = _prepare(
            (A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0), dtype)
        r0c = _prepare((r0,), dtype)[0] if r0 is not None else None
        rtc = _prepare((r_traj,), dtype)[0] if r_traj is not None else None
        f32 = dict(device=dev, dtype=torch.float32)
        u_traj = torch.empty(N, nh, T, du, device=dev, dtype=dtype)
        states = torch.empty(N, nh, T, d, **f32) if return_states else None
        costates = torch.empty(N, nh, T, d, **f32) if return_costates else None
        lam0_out = torch.empty(N, nh, d, **f32) if return_lambda0 else None
        cost = torch.empty(N, nh, **f32) if return_cost else None
        per_row = nh * d * du * 4
        rows = N if r0 is None else max(1, min(N, budget // per_row))
        lib = _lib.load()
        u1 = torch.empty(min(rows, N), nh, du, device=dev, dtype=dtype)
        lam0 = torch.empty(min(rows, N), nh, d, **f32)
        M = torch.empty(min(rows, N), nh, d, du, **f32) if r0 is not None else None
        status = torch.zeros(2, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev):
            for a in range(0, N, rows):
                n = min(rows, N - a)
                sl = lambda t: None if t is None else t[a:a + n]  # noqa: E731
                ins = [sl(t) for t in (A, Bm, Qm, R, Qf, lA, lB, lQ, H0)]
                if rtc is not None:
                    _launch("ttc_lqr_fwd_affine", dev, lib.ttc_lqr_fwd_affine, *[_ptr(t) for t in ins],
                            _ptr(sl(rtc)), n, nh, d, du, T, _DTYPES[dtype], _flags(inv_guard), _ptr(u1),
                            _ptr(lam0), _ptr(status[0:1]))
                else:
                    _launch("ttc_lqr_fwd", dev, lib.ttc_lqr_fwd, *[_ptr(t) for t in ins], n, nh, d, du,
                            T, _DTYPES[dtype], _flags(inv_guard), _ptr(u1), _ptr(lam0), _ptr(M),
                            _ptr(status[0:1]))
                r, r_steps = (sl(rtc), T) if rtc is not None else (sl(r0c), 1)
                _launch("ttc_lqr_rollout", dev, lib.ttc_lqr_rollout, *[_ptr(t) for t in ins],
                        _ptr(lam0), _ptr(M), _ptr(r), r_steps, n, nh, d, du, T, _DTYPES[dtype],
                        _ptr(sl(u_traj)), _ptr(sl(states)), _ptr(sl(costates)), _ptr(sl(lam0_out)),
                        _ptr(sl(cost)), _ptr(status[1:2]))
        st = status.tolist()
        check_fwd_status(st[0])
        if st[1] & _lib.STATUS_TRAJ_NONFINITE:
            raise RuntimeError(TRAJ_NONFINITE_MSG)
    extra = [t for t, want in ((states, return_states), (costates, return_costates),
                               (lam0_out, return_lambda0), (cost, return_cost)) if want]
    return (u_traj, *extra) if extra else u_traj
