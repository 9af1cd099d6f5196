"""CPU oracle for TTC-Net's LQR hot path -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and the ``--impl reference`` arm) may import this module, and only as the
checker or as the timed CPU baseline.  The product package ``ttc_b200`` never
imports it; the CUDA path fails loudly instead of falling back to it.

It restates, in plain PyTorch on the CPU (fp32 or fp64), the algorithms of the
reference implementation VITA-Group/TTC-Net (``ttc/`` package):

* ``l2norm``                 -- fla ``l2norm`` (fla/modules/l2norm.py:42, third-party
                                 dependency pinned by the reference at fla==0.3.1)
* ``time_varying_system``    -- ttc/solvers/torch_lqr.py:65-91  (_generate_parameters)
* ``riccati_actions``        -- ttc/solvers/lin_solver_lqr.py:113-212 (solve_traj_actions)
* ``traj_states``            -- ttc/solvers/lin_solver_lqr.py:13-110  (solve_traj_states)
* ``riccati_solve``          -- ttc/solvers/torch_lqr.py:93-118 (direct_lqr_solve, "riccati")
* ``kkt_solve``              -- ttc/solvers/torch_lqr.py:12-63,120-139 ("kkt")
* ``fused_forward``          -- ttc/solvers/fused_lqr.py:18-146 with the Triton kernels
                                 symplectic_iter.py:207-300 (rev_iter) and :415-517
                                 (dec_first_step)
* ``fused_backward``         -- ttc/solvers/fused_lqr.py:148-253 with
                                 symplectic_iter.py:715-885 (fwd_iter_diff)
* ``fused_solve``            -- ttc/solvers/fused_lqr.py:255-304 ("fused")
* ``TTCLayerOracle``         -- ttc/layers/ttc_layer.py:24-153

Parity pin: ``tests/test_oracle_golden.py`` checks every function above against
golden vectors that ``tests/golden/make_golden.py`` produced by running the
reference package itself (riccati and kkt solvers, TTCLayer) in the build
container.  The Triton ``fused`` solver needs a GPU and Triton and could not be
run there; its restatement here is pinned through the kkt backward, which uses
the same symmetrised Q/Q_f gradient convention.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = [
    "l2norm", "time_varying_system", "riccati_actions", "traj_states",
    "riccati_solve", "kkt_solve", "fused_forward", "fused_backward",
    "fused_solve", "TTCLayerOracle", "SOLVERS", "max_rel",
]


def max_rel(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max|out-ref| / max|ref| -- the per-tensor error measure used by every parity test."""
    out = out.detach().double()
    ref = ref.detach().double()
    den = ref.abs().max().item()
    num = (out - ref).abs().max().item()
    if den == 0.0:
        return num
    return num / den


# ---------------------------------------------------------------------------
# fla l2norm (third-party, restated)
# ---------------------------------------------------------------------------
def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = x / sqrt(sum(x^2) + eps) over the last dim, computed in at least fp32
    and cast back to x.dtype (fla/modules/l2norm.py:42 forward kernel; its
    backward :69 is the exact derivative of this expression, so autograd through
    it reproduces fla's l2norm_bwd)."""
    work = torch.promote_types(x.dtype, torch.float32)
    xf = x.to(work)
    y = xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)
    return y.to(x.dtype)


# ---------------------------------------------------------------------------
# Time-varying LQR system (riccati / kkt semantics)
# ---------------------------------------------------------------------------
def time_varying_system(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, T):
    """Expand the per-problem parameters over the horizon (torch_lqr.py:65-91).

    For exponents t = 1..T:
      A_t = 1 + A_diag * exp(lgA * t)                       [N,nh,T,d]
      B_t = B * diag(exp(lgB * t))                          [N,nh,T,d,du]
      Q list index k = 0..T-2 carries exponent k+1:
        Q_k = diag(exp(lgQ*(k+1))) Q diag(exp(lgQ*(k+1))),  and index T-1 is Q_f
      R_t = 1 / R_inv                                       [N,nh,T,du]
    """
    N, nh, d = A_diag.shape
    du = B.shape[-1]
    t = torch.arange(1, T + 1, dtype=A_diag.dtype, device=A_diag.device)
    gA = torch.exp(log_gamma_A[..., None] * t)                         # [N,nh,T]
    A_t = 1.0 + A_diag[:, :, None, :] * gA[..., None]                  # [N,nh,T,d]
    gB = torch.exp(log_gamma_B[:, :, None, :] * t[:, None])            # [N,nh,T,du]
    B_t = B[:, None, None, :, :] * gB[:, :, :, None, :]                # [N,nh,T,d,du]
    gQ = torch.exp(log_gamma_Q[:, :, None, :] * t[:-1, None])          # [N,nh,T-1,d]
    Q_t = gQ[..., :, None] * Q[:, None, None, :, :] * gQ[..., None, :]  # [N,nh,T-1,d,d]
    Q_t = torch.cat([Q_t, Q_f[:, :, None, :, :]], dim=2)              # [N,nh,T,d,d]
    R_t = (1.0 / R_inv)[:, :, None, :].expand(N, nh, T, du)
    return A_t, B_t, Q_t, R_t


def riccati_actions(A_t, B_t, Q_t, R_t, h0, r_traj=None, return_traj=False,
                    solve_dtype=torch.float32):
    """Finite-horizon LQR by the backward Riccati sweep (lin_solver_lqr.py:113-212).

    Shapes (M independent problems): A_t [M,T,d] (diagonal), B_t [M,T,d,du],
    Q_t [M,T,d,d] (index k is the stage cost of state h_{k+1}; index T-1 is the
    terminal cost), R_t [M,T,du] (diagonal), h0 [M,d], r_traj [M,T,du] or None.

    Stage t has cost blocks [[Qs_t, 0], [0, R_t]] with Qs_0 = 0 and Qs_t = Q_t[t-1]
    (lin_solver_lqr.py:137-139); the value recursion starts from V = Q_t[T-1]
    (:148).  The gain solves run in ``solve_dtype`` (the reference casts Quu to
    fp32, :175-177); pass None to solve in the working dtype.

    Returns u_0 [M,du], or the closed-loop action trajectory [M,T,du] when
    ``return_traj`` (rollout :187-203).
    """
    M_, T, d = A_t.shape
    du = B_t.shape[-1]
    dt = Q_t.dtype
    V = Q_t[:, T - 1]
    v = torch.zeros(M_, d, dtype=dt, device=h0.device)
    Ks = [None] * T
    ks = [None] * T
    for t in range(T - 1, -1, -1):
        a = A_t[:, t]                                   # [M,d]
        Bm = B_t[:, t]                                  # [M,d,du]
        VA = V * a[:, None, :]                          # V diag(a)
        Qxx = a[:, :, None] * VA                        # diag(a) V diag(a)
        if t >= 1:
            Qxx = Qxx + Q_t[:, t - 1]
        VB = V @ Bm                                     # [M,d,du]
        Qxu = a[:, :, None] * VB                        # diag(a) V B
        Qux = Bm.transpose(-1, -2) @ VA                 # B^T V diag(a)
        Quu = Bm.transpose(-1, -2) @ VB + torch.diag_embed(R_t[:, t])
        qx = a * v
        qu = (Bm.transpose(-1, -2) @ v[..., None])[..., 0]
        if r_traj is not None:
            qu = qu + r_traj[:, t]
        sd = dt if solve_dtype is None else solve_dtype
        Quu_s = Quu.to(sd)
        K = -torch.linalg.solve(Quu_s, Qux.to(sd)).to(dt)                 # [M,du,d]
        k = -torch.linalg.solve(Quu_s, qu[..., None].to(sd))[..., 0].to(dt)  # [M,du]
        Ks[t], ks[t] = K, k
        KT = K.transpose(-1, -2)
        V = Qxx + Qxu @ K + KT @ Qux + KT @ Quu @ K
        v = qx + (Qxu @ k[..., None])[..., 0] + (KT @ qu[..., None])[..., 0] \
            + (KT @ (Quu @ k[..., None]))[..., 0]
    if not return_traj:
        return (Ks[0] @ h0[..., None])[..., 0] + ks[0]
    u_traj = torch.zeros(M_, T, du, dtype=dt, device=h0.device)
    x = h0
    for t in range(T):
        u = (Ks[t] @ x[..., None])[..., 0] + ks[t]
        u_traj[:, t] = u
        if t < T - 1:
            x = A_t[:, t] * x + (B_t[:, t] @ u[..., None])[..., 0]
    return u_traj


def traj_states(u_traj, A_t, B_t, Q_t, h0):
    """Roll out states and costates for a given action trajectory
    (lin_solver_lqr.py:13-110).

    states[:, t] = h_{t+1} = A_t h_t + B_t u_t;  costates[:, t] = lambda_{t+1} with
    lambda_T = Q_t[T-1] h_T and lambda_{t+1} = Q_t[t] h_{t+1} + A_{t+1} lambda_{t+2};
    lambda_0 = A_0 lambda_1.  h0 None means a zero initial state.
    Returns (states [M,T,d], costates [M,T,d], lambda0 [M,d]).
    """
    M_, T, d = A_t.shape
    x = torch.zeros(M_, d, dtype=A_t.dtype) if h0 is None else h0
    states = []
    for t in range(T):
        x = A_t[:, t] * x + (B_t[:, t] @ u_traj[:, t][..., None])[..., 0]
        states.append(x)
    states = torch.stack(states, dim=1)
    cost = [None] * T
    cost[T - 1] = (Q_t[:, T - 1] @ states[:, T - 1][..., None])[..., 0]
    for t in range(T - 2, -1, -1):
        cost[t] = (Q_t[:, t] @ states[:, t][..., None])[..., 0] + A_t[:, t + 1] * cost[t + 1]
    costates = torch.stack(cost, dim=1)
    lam0 = A_t[:, 0] * costates[:, 0]
    return states, costates, lam0


def traj_cost(u_traj, states, Q_t, R_t, r_traj=None):
    """Total cost of a trajectory (lin_solver_lqr.py:55-68):
    sum_t 0.5 h_{t+1}^T Q_t h_{t+1} + 0.5 u_t^T diag(R_t) u_t + r_t^T u_t.  Returns [M]."""
    qh = (Q_t @ states[..., None])[..., 0]
    c = 0.5 * (states * qh).sum(-1) + 0.5 * (u_traj * R_t * u_traj).sum(-1)
    if r_traj is not None:
        c = c + (r_traj * u_traj).sum(-1)
    return c.sum(-1)


def _flat(A_t, B_t, Q_t, R_t):
    N, nh, T, d = A_t.shape
    du = B_t.shape[-1]
    return (A_t.reshape(-1, T, d), B_t.reshape(-1, T, d, du),
            Q_t.reshape(-1, T, d, d), R_t.reshape(-1, T, du))


def riccati_solve(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                  solve_dtype=torch.float32):
    """The reference "riccati" solver (torch_lqr.py:93-118); differentiable by autograd."""
    N, nh, d = A_diag.shape
    du = B.shape[-1]
    A_t, B_t, Q_t, R_t = _flat(*time_varying_system(
        A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, T))
    u = riccati_actions(A_t, B_t, Q_t, R_t, h0.reshape(-1, d), solve_dtype=solve_dtype)
    return u.reshape(N, nh, du)


class _KKTFunc(torch.autograd.Function):
    """KKT adjoint of the LQR solve (torch_lqr.py:12-63): the backward solves a second
    LQR driven by the affine action cost r_0 = du, rolls out states/costates of both
    problems and forms outer-product gradients w.r.t. the time-varying system."""

    @staticmethod
    def forward(ctx, A_t, B_t, Q_t, R_t, h0):
        u = riccati_actions(A_t, B_t, Q_t, R_t, h0)
        ctx.save_for_backward(h0, A_t, B_t, Q_t, R_t)
        return u

    @staticmethod
    def backward(ctx, d_u):
        h0, A_t, B_t, Q_t, R_t = ctx.saved_tensors
        M_, T, d = A_t.shape
        du = B_t.shape[-1]
        r = torch.zeros(M_, T, du, dtype=A_t.dtype)
        r[:, 0] = d_u
        u_f = riccati_actions(A_t, B_t, Q_t, R_t, h0, return_traj=True)
        u_b = riccati_actions(A_t, B_t, Q_t, R_t, torch.zeros_like(h0), r_traj=r,
                              return_traj=True)
        hs_f, lam_f, _ = traj_states(u_f, A_t, B_t, Q_t, h0)
        hs_b, lam_b, lam0_b = traj_states(u_b, A_t, B_t, Q_t, None)
        hs_f_prev = torch.cat([h0[:, None], hs_f[:, :-1]], dim=1)
        hs_b_prev = torch.cat([torch.zeros_like(h0)[:, None], hs_b[:, :-1]], dim=1)
        gA = hs_f_prev * lam_b + hs_b_prev * lam_f
        gB = lam_b[..., :, None] * u_f[..., None, :] + lam_f[..., :, None] * u_b[..., None, :]
        gQ = (hs_b[..., :, None] * hs_f[..., None, :] + hs_f[..., :, None] * hs_b[..., None, :]) / 2.0
        gR = u_f * u_b
        return gA, gB, gQ, gR, lam0_b


def kkt_solve(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T):
    """The reference "kkt" solver (torch_lqr.py:120-139): riccati forward, KKT backward."""
    N, nh, d = A_diag.shape
    du = B.shape[-1]
    A_t, B_t, Q_t, R_t = _flat(*time_varying_system(
        A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, T))
    u = _KKTFunc.apply(A_t, B_t, Q_t, R_t, h0.reshape(-1, d))
    return u.reshape(N, nh, du)


# ---------------------------------------------------------------------------
# Fused (symplectic) solver restatement
# ---------------------------------------------------------------------------
def fused_forward(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                  normalize_threshold: float = 1e3, inv_guard: bool = False, r_traj=None):
    """Symplectic Riccati sweep + LU solve + first-step decode (fused_lqr.py:18-146).

    Y1 = I, Y2 = Q_f (fused_lqr.py:50-52); for s = 0..T-1 with tau = T-s (A/B
    exponent) and tq = T-1-s (Q exponent)  (symplectic_iter.py:207-209,262-264):
        Y2BR = (Y2 B_tau) diag(R_inv)                              (:230-232)
        Y1   = (Y1 + Y2BR B_tau^T) diag(A_tau)^-1                  (:233,246-252)
        Y2   = Y2 diag(A_tau) + Y1 Q_tq   (s < T-1),  Y2 diag(A_tau) (s = T-1)  (:254-259)
        at s = T-1: Y3 = -Y2BR                                      (:241-243)
        normalisation NORMALIZE_TYPE=2: divide Y1, Y2 (and Y3 at the last step) by the
        largest row abs-sum of Y1 or Y2 when it exceeds 1e3          (:286-300)
    The oracle normalises the whole d x d block (the reference's BY = d tiling).
    inv_guard adds 1e-6 I to the final Y1 (INV_GUARD, symplectic_iter.py:302-305).
    P = Y1^-1 Y2 (LU, :104-105); lambda0 = P h0; lambda1 = lambda0 / (1 + A_diag e^lgA);
    u = -R_inv * (B diag(e^lgB))^T lambda1 (symplectic_iter.py:437,472-517).
    Returns u, lam0, Y1, Y2, Y3, P (all in the working dtype).

    r_traj [N,nh,T,du]: an affine action cost r_t^T u_t on every step (the restatement of the
    CUDA path's per-step affine forward, not a reference kernel).  Row i of the sweep is the
    constraint Y1_i . lambda = Y2_i . h + c_i; each step adds c -= Y2BR r_{T-1-s} (Y2BR of
    the step, before Y2's update) and the normalisation divides c with its rows.  Then
    lambda0 = Y1^-1 (Y2 h0 + c) and u gets -R_inv r_0; with r_traj zero after step 0,
    c = Y3 r_0, the IS_AFFINE y3 (symplectic_iter.py:211-243).
    """
    N, nh, d = A_diag.shape
    dt = Q_f.dtype
    Y1 = torch.eye(d, dtype=dt).expand(N, nh, d, d).clone()
    Y2 = Q_f.clone()
    Bh = B[:, None]
    Qh = Q[:, None]
    Y3 = None
    c = None if r_traj is None else torch.zeros(N, nh, d, dtype=dt)
    for s in range(T):
        tau = float(T - s)
        tq = float(T - 1 - s)
        Bt = Bh * torch.exp(log_gamma_B * tau)[:, :, None, :]
        Y2BR = (Y2 @ Bt) * R_inv[:, :, None, :]
        if c is not None:
            c = c - (Y2BR @ r_traj[:, :, T - 1 - s, :, None])[..., 0]
        Y1 = Y1 + Y2BR @ Bt.transpose(-1, -2)
        At = 1.0 + A_diag * torch.exp(log_gamma_A * tau)[..., None]
        Y1 = Y1 / At[:, :, None, :]
        if s < T - 1:
            e = torch.exp(log_gamma_Q * tq)
            Qt = e[..., :, None] * Qh * e[..., None, :]
            Y2 = Y2 * At[:, :, None, :] + Y1 @ Qt
        else:
            Y2 = Y2 * At[:, :, None, :]
            Y3 = -Y2BR
        m = torch.maximum(Y1.abs().sum(-1).amax(-1), Y2.abs().sum(-1).amax(-1))
        sc = torch.where(m > normalize_threshold, m, torch.ones_like(m))[..., None, None]
        Y1 = Y1 / sc
        Y2 = Y2 / sc
        if c is not None:
            c = c / sc[..., 0]
        if s == T - 1:
            Y3 = Y3 / sc
    if inv_guard:
        Y1 = Y1 + 1e-6 * torch.eye(d, dtype=dt)
    P = torch.linalg.solve(Y1, Y2)
    lam0 = (P @ h0[..., None])[..., 0]
    if c is not None:
        lam0 = torch.linalg.solve(Y1, (Y2 @ h0[..., None])[..., 0] + c)
    lam1 = lam0 / (1.0 + A_diag * torch.exp(log_gamma_A)[..., None])
    B1 = Bh * torch.exp(log_gamma_B)[:, :, None, :]
    u = -R_inv * (B1.transpose(-1, -2) @ lam1[..., None])[..., 0]
    if c is not None:
        u = u - R_inv * r_traj[:, :, 0]
    return u, lam0, Y1, Y2, Y3, P


def fused_backward(A_diag, B, Q, R_inv, log_gamma_A, log_gamma_B, log_gamma_Q, h0, lam0,
                   Y1, Y3, d_u, T):
    """Forward-in-time adjoint integration (fused_lqr.py:182-253 and
    symplectic_iter.py:715-885).  Returns the 9 gradients
    (A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0) in the working dtype.

    d_p = Y1^-1 (Y3 du)  (fused_lqr.py:185-187); state (h, dh, lam, dlam) starts at
    (h0, 0, lambda0, d_p).  For step k = 0..T-1 (A/B exponent e = k+1, Q exponent k
    at the top of the step and k+1 after the state update):
      k > 0: lam -= Q_k h, dlam -= Q_k dh                        (:766-775)
      k = 0: grad_h0 = dlam                                      (:777-779)
      lam, dlam /= A_e; dA = lam dh + dlam h                     (:781-798)
      u = -R_inv B_e^T lam, du = -R_inv B_e^T dlam (k=0: du -= R_inv d_u)  (:800-823)
      dB = lam du^T + dlam u^T                                   (:826-835)
      h = A_e h + B_e u, dh = A_e dh + B_e du                    (:838-845)
      dQ = (h dh^T + dh h^T)/2 -> grad_Qf (k = T-1) or grad_Q, grad_lgQ  (:855-877)
      grad_R_inv += -(u du) / R_inv^2                            (:880-883)
    grad_B and grad_Q are summed over heads (the reference's gpu-scope atomics).
    """
    N, nh, d = A_diag.shape
    d_p = torch.linalg.solve(Y1, (Y3 @ d_u[..., None]))[..., 0]
    g_A = torch.zeros_like(A_diag)
    g_B = torch.zeros_like(B)
    g_Q = torch.zeros_like(Q)
    g_R = torch.zeros_like(R_inv)
    g_Qf = None
    g_lgA = torch.zeros_like(log_gamma_A)
    g_lgB = torch.zeros_like(log_gamma_B)
    g_lgQ = torch.zeros_like(log_gamma_Q)
    g_h0 = None
    h = h0.clone()
    dh = torch.zeros_like(h0)
    lam = lam0.clone()
    dlam = d_p.clone()
    Bh = B[:, None]
    Qh = Q[:, None]
    for k in range(T):
        if k > 0:
            e = torch.exp(log_gamma_Q * float(k))
            Qt = e[..., :, None] * Qh * e[..., None, :]
            lam = lam - (Qt @ h[..., None])[..., 0]
            dlam = dlam - (Qt @ dh[..., None])[..., 0]
        if k == 0:
            g_h0 = dlam.clone()
        ea = torch.exp(log_gamma_A * float(k + 1))[..., None]
        At = 1.0 + A_diag * ea
        lam = lam / At
        dlam = dlam / At
        dA = lam * dh + dlam * h
        g_A = g_A + dA * ea
        g_lgA = g_lgA + (dA * A_diag).sum(-1) * float(k + 1) * ea[..., 0]
        eb = torch.exp(log_gamma_B * float(k + 1))
        Bt = Bh * eb[:, :, None, :]
        u = -R_inv * (Bt.transpose(-1, -2) @ lam[..., None])[..., 0]
        du = -R_inv * (Bt.transpose(-1, -2) @ dlam[..., None])[..., 0]
        if k == 0:
            du = du - d_u * R_inv
        dB = lam[..., :, None] * du[..., None, :] + dlam[..., :, None] * u[..., None, :]
        g_B = g_B + (dB * eb[:, :, None, :]).sum(1)
        g_lgB = g_lgB + (dB * Bh).sum(-2) * float(k + 1) * eb
        h = h * At + (Bt @ u[..., None])[..., 0]
        dh = dh * At + (Bt @ du[..., None])[..., 0]
        dQ = (h[..., :, None] * dh[..., None, :] + dh[..., :, None] * h[..., None, :]) / 2.0
        if k == T - 1:
            g_Qf = dQ
        else:
            e = torch.exp(log_gamma_Q * float(k + 1))
            g_Q = g_Q + (e[..., :, None] * dQ * e[..., None, :]).sum(1)
            g_lgQ = g_lgQ + ((dQ * Qh * e[..., :, None]).sum(-2)
                             + (dQ * Qh * e[..., None, :]).sum(-1)) * float(k + 1) * e
        g_R = g_R - (u * du) / (R_inv * R_inv)
    return g_A, g_B, g_Q, g_R, g_Qf, g_lgA, g_lgB, g_lgQ, g_h0


class _FusedFunc(torch.autograd.Function):
    """Autograd wrapper of the fused restatement (fused_lqr.py:255-291)."""

    @staticmethod
    def forward(ctx, A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T, inv_guard=False):
        u, lam0, Y1, _, Y3, _ = fused_forward(A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T,
                                              inv_guard=inv_guard)
        ctx.save_for_backward(A_diag, B, Q, R_inv, lgA, lgB, lgQ, h0, lam0, Y1, Y3)
        ctx.T = T
        return u

    @staticmethod
    def backward(ctx, d_u):
        A_diag, B, Q, R_inv, lgA, lgB, lgQ, h0, lam0, Y1, Y3 = ctx.saved_tensors
        g = fused_backward(A_diag, B, Q, R_inv, lgA, lgB, lgQ, h0, lam0, Y1, Y3, d_u, ctx.T)
        return (*g, None, None)


def fused_solve(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                inv_guard: bool = False):
    """The reference "fused" solver semantics on the CPU (fused_lqr.py:294-304)."""
    return _FusedFunc.apply(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                            inv_guard)


SOLVERS = {"riccati": riccati_solve, "kkt": kkt_solve, "fused": fused_solve}


# ---------------------------------------------------------------------------
# Trajectories (solve_traj_actions(return_traj=True) + solve_traj_states)
# ---------------------------------------------------------------------------
def riccati_trajectory(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                       r_traj=None, solve_dtype=torch.float32):
    """Closed-loop trajectory by the backward Riccati sweep and its rollout
    (lin_solver_lqr.py:113-212 with return_traj=True), then states, costates, lambda0 and
    total cost (solve_traj_states, lin_solver_lqr.py:13-110), on the time-varying system of
    torch_lqr.py:65-91.  r_traj [N,nh,T,du] or None.
    Returns (u_traj [N,nh,T,du], states [N,nh,T,d], costates [N,nh,T,d], lambda0 [N,nh,d],
    cost [N,nh])."""
    N, nh, d = A_diag.shape
    du = B.shape[-1]
    A_t, B_t, Q_t, R_t = _flat(*time_varying_system(
        A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, T))
    r = None if r_traj is None else r_traj.reshape(-1, T, du)
    u = riccati_actions(A_t, B_t, Q_t, R_t, h0.reshape(-1, d), r_traj=r, return_traj=True,
                        solve_dtype=solve_dtype)
    hs, lam, lam0 = traj_states(u, A_t, B_t, Q_t, h0.reshape(-1, d))
    cost = traj_cost(u, hs, Q_t, R_t, r)
    return (u.reshape(N, nh, T, du), hs.reshape(N, nh, T, d), lam.reshape(N, nh, T, d),
            lam0.reshape(N, nh, d), cost.reshape(N, nh))


def fused_trajectory(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                     r0=None, inv_guard: bool = False, r_traj=None):
    """The trajectory as the CUDA path computes it: the symplectic forward (fused_forward)
    gives lambda0 = P h0 and M = Y1^-1 Y3; an affine action cost r0 [N,nh,du] on step 0 adds
    M r0 to lambda0 (Y1^-1 y3 with the y3 = Y3 r of the reference's IS_AFFINE sweep,
    symplectic_iter.py:211-238) and -R_inv r0 to u_0.  State and costate are then integrated
    forward in time as in the primal half of the reference's adjoint
    (symplectic_iter.py:766-845; the same recursion as fused_backward):
        k > 0: lam -= Q_k h;  lam /= A_{k+1};  u_k = -R_inv B_{k+1}^T lam;  h = A_{k+1} h + B_{k+1} u_k
    r_traj [N,nh,T,du] (instead of r0): an affine cost on every step; lambda0 from
    fused_forward(r_traj=...) and u_k -= R_inv r_k on every step.
    Returns (u_traj, states, costates, lambda0, cost) as riccati_trajectory."""
    N, nh, d = A_diag.shape
    du = B.shape[-1]
    _, lam, Y1, _, Y3, _ = fused_forward(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B,
                                         log_gamma_Q, h0, T, inv_guard=inv_guard, r_traj=r_traj)
    if r0 is not None:
        lam = lam + torch.linalg.solve(Y1, Y3 @ r0[..., None])[..., 0]
    lam0 = lam
    h = h0
    Bh, Qh = B[:, None], Q[:, None]
    us, hs, ls = [], [], []
    cost = torch.zeros(N, nh, dtype=A_diag.dtype)
    for k in range(T):
        if k > 0:
            e = torch.exp(log_gamma_Q * float(k))
            qh = (e[..., :, None] * Qh * e[..., None, :] @ h[..., None])[..., 0]
            lam = lam - qh
            cost = cost + 0.5 * (h * qh).sum(-1)
        At = 1.0 + A_diag * torch.exp(log_gamma_A * float(k + 1))[..., None]
        lam = lam / At
        Bt = Bh * torch.exp(log_gamma_B * float(k + 1))[:, :, None, :]
        u = -R_inv * (Bt.transpose(-1, -2) @ lam[..., None])[..., 0]
        rk = r0 if k == 0 else None
        if r_traj is not None:
            rk = r_traj[:, :, k]
        if rk is not None:
            u = u - R_inv * rk
            cost = cost + (rk * u).sum(-1)
        cost = cost + 0.5 * (u * u / R_inv).sum(-1)
        h = h * At + (Bt @ u[..., None])[..., 0]
        us.append(u)
        hs.append(h)
        ls.append(lam)
    cost = cost + 0.5 * (h * (Q_f @ h[..., None])[..., 0]).sum(-1)
    return torch.stack(us, 2), torch.stack(hs, 2), torch.stack(ls, 2), lam0, cost


# ---------------------------------------------------------------------------
# Layer
# ---------------------------------------------------------------------------
class TTCLayerOracle(nn.Module):
    """CPU restatement of TTCLayer (ttc/layers/ttc_layer.py:24-153), same parameter names
    and shapes (``in_proj``, ``out_proj``, ``Bs``, ``Qs``, ``bias_gamma``) so a state_dict
    moves 1:1 between this class, the reference and ``ttc_b200.TTCLayer``."""

    def __init__(self, in_dim, out_dim, h_dim, num_heads, b_rank, q_rank, u_dim=None,
                 bias=False, gamma_bias=False, gamma_bias_init="sqrt_dim",
                 rescale="l2_norm", q_reparam="plain", solver_impl="riccati"):
        super().__init__()
        u_dim = h_dim if u_dim is None else u_dim
        assert solver_impl in SOLVERS, f"Unknown LQR solver {solver_impl}"
        assert rescale in ("none", "l2_norm", "h0_norm")
        assert q_reparam in ("plain", "cholesky")
        assert gamma_bias_init in ("sqrt_dim", "zero")
        self.solver = SOLVERS[solver_impl]
        self.rescale, self.q_reparam = rescale, q_reparam
        self.in_dim, self.out_dim, self.num_heads = in_dim, out_dim, num_heads
        self.h_dim, self.u_dim, self.q_rank, self.b_rank = h_dim, u_dim, q_rank, b_rank
        width = (4 * h_dim + 2 * u_dim + 1) * num_heads + b_rank + q_rank
        self.in_proj = nn.Linear(in_dim, width, bias=bias)
        self.out_proj = nn.Linear(u_dim * num_heads, out_dim, bias=bias)
        self.Bs = nn.Parameter(torch.empty(b_rank, h_dim, u_dim))
        self.Qs = nn.Parameter(torch.empty(q_rank, h_dim, h_dim))
        self.bias_gamma = None
        if gamma_bias:
            self.bias_gamma = nn.Parameter(torch.empty(1 + u_dim + h_dim, dtype=torch.float32))
        with torch.no_grad():
            self.Bs.normal_(0.0, 0.02)
            if q_reparam == "plain":
                g = torch.empty_like(self.Qs).normal_(0.0, 0.02)
                self.Qs.copy_(g @ g.transpose(1, 2) / math.sqrt(h_dim))
            else:
                self.Qs.normal_(0.0, 0.02)
            if self.bias_gamma is not None:
                fill = math.log(1.0 / math.sqrt(h_dim)) if gamma_bias_init == "sqrt_dim" else 0.0
                self.bias_gamma.fill_(fill)

    def solver_inputs(self, x2d):
        """Prologue (ttc_layer.py:104-135): x [rows, in_dim] -> the 9 solver inputs."""
        nh, d, du = self.num_heads, self.h_dim, self.u_dim
        z = self.in_proj(x2d)
        heads, cB, cQ = torch.split(z, [(4 * d + 2 * du + 1) * nh, self.b_rank, self.q_rank], -1)
        h0, A, Rr, cQf, lg = torch.split(heads.view(-1, nh, 4 * d + 2 * du + 1),
                                         [d, d, du, d, 1 + du + d], -1)
        A = l2norm(A)
        cB, cQ, cQf = l2norm(cB), l2norm(F.softplus(cQ)), l2norm(F.softplus(cQf))
        Bm = torch.einsum("...r,rmn->...mn", cB, self.Bs)
        if self.q_reparam == "plain":
            Qm = torch.einsum("...r,rmn->...mn", cQ, self.Qs)
            Qf = torch.einsum("...r,rmn->...mn", cQf, self.Qs)
        else:
            Qm = torch.einsum("...r,rmn,rkn->...mk", cQ, self.Qs, self.Qs) / math.sqrt(d)
            Qf = torch.einsum("...r,rmn,rkn->...mk", cQf, self.Qs, self.Qs) / math.sqrt(d)
        Rinv = torch.clamp(l2norm(F.softplus(Rr)), min=1e-6)
        if self.bias_gamma is not None:
            lg = -F.softplus(lg) - F.relu(-self.bias_gamma[None, None, :])
        else:
            lg = -F.softplus(lg)
        lgA, lgB, lgQ = torch.split(lg, [1, du, d], -1)
        return A, Bm, Qm, Rinv, Qf, lgA.squeeze(-1), lgB, lgQ, h0

    def forward(self, x, T: int):
        """ttc_layer.py:98-153 on x [bs, seq, in_dim] -> y [bs, seq, out_dim]."""
        if T == 0:
            return torch.zeros(x.shape[0], x.shape[1], self.out_dim, dtype=x.dtype)
        bs, seq, in_dim = x.shape
        args = self.solver_inputs(x.reshape(-1, in_dim))
        u = self.solver(*args, T)
        if torch.isnan(u).any():
            raise RuntimeError("NaN detected in TTC layer solver output.")
        if self.rescale == "l2_norm":
            u = l2norm(u)
        elif self.rescale == "h0_norm":
            h0 = args[-1]
            h0n = torch.linalg.norm(h0, dim=-1, ord=2).detach()
            un = torch.linalg.norm(u, dim=-1, ord=2).detach()
            u = u / un[..., None] * h0n[..., None]
        return self.out_proj(u.reshape(bs, seq, -1))
