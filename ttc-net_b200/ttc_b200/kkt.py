"""``solver_impl="kkt"`` on the GPU: the reference's kkt solver over the B200 kernels.

The reference's kkt solver (ttc/solvers/torch_lqr.py:12-63,120-139) returns the Riccati
action u_0 and, in its backward, solves a second LQR driven by the affine action cost
r_0 = du (zero initial state), rolls out states and costates of both problems and forms
outer-product gradients with respect to the time-varying system of ``_generate_parameters``
(torch_lqr.py:65-91), which autograd then carries to the nine solver inputs.

Here the forward is ``ttc_lqr_fwd`` (the same u).  The backward runs one more
``ttc_lqr_fwd`` (lambda0 = P h0 and M = Y1^-1 Y3, shared by both problems: the second one's
lambda0 is M du) and two ``ttc_lqr_rollout`` launches, then forms the reference's gradients
(torch_lqr.py:49-61) and their chain rule through the time-varying system in closed form, as
contractions over heads and steps: no [.., T, d, d] tensor is built.  The gradients use the
symmetrised Q / Q_f convention of the reference's kkt and fused backward.  Work and state are
fp32 whatever the activation dtype (the reference's kkt buffers are fp32 only); gradients are
cast back to each input's dtype.
"""
from __future__ import annotations

import torch

from . import _lib
from .solver import (SAVE_BUDGET_BYTES, _DTYPES, _check_shapes, _launch, _prepare, _ptr,
                     check_fwd_status)
from .trajectory import TRAJ_NONFINITE_MSG

_F32 = _DTYPES[torch.float32]
# Device memory the backward's trajectories and gradient temporaries may take at once, and
# the bytes they take per row, head, step and vector entry (six fp32 trajectories plus the
# gradient terms formed from them, about three times that).
KKT_WORK_BYTES = 16 << 30
KKT_BYTES_PER_STEP = 12


def _rollouts(args, T, d_u, budget):
    """Both problems of the kkt backward on the prepared fp32 inputs: (u, states, costates)
    of the forward problem and of the one with h0 = 0 and the affine cost d_u on step 0, plus
    the latter's lambda0."""
    A, Bm, Qm, R, Qf, lA, lB, lQ, H0 = args
    N, nh, d = A.shape
    du = Bm.shape[-1]
    dev = A.device
    f32 = dict(device=dev, dtype=torch.float32)
    out_f = [torch.empty(N, nh, T, du, **f32), torch.empty(N, nh, T, d, **f32),
             torch.empty(N, nh, T, d, **f32)]
    out_b = [torch.empty(N, nh, T, du, **f32), torch.empty(N, nh, T, d, **f32),
             torch.empty(N, nh, T, d, **f32)]
    lam0_b = torch.empty(N, nh, d, **f32)
    rows = max(1, min(N, budget // (nh * d * du * 4)))
    u1 = torch.empty(rows, nh, du, **f32)
    lam0 = torch.empty(rows, nh, d, **f32)
    M = torch.empty(rows, nh, d, du, **f32)
    zeros = torch.zeros(rows, nh, d, **f32)
    status = torch.zeros(2, device=dev, dtype=torch.int32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        for a in range(0, N, rows):
            n = min(rows, N - a)
            ins = [t[a:a + n] for t in args]
            _launch("ttc_lqr_fwd", dev, lib.ttc_lqr_fwd, *[_ptr(t) for t in ins], n, nh, d, du, T,
                    _F32, 0, _ptr(u1), _ptr(lam0), _ptr(M), _ptr(status[0:1]))
            # forward problem: lambda0 = P h0
            _launch("ttc_lqr_rollout", dev, lib.ttc_lqr_rollout, *[_ptr(t) for t in ins], _ptr(lam0),
                    None, None, 1, n, nh, d, du, T, _F32, *[_ptr(o[a:a + n]) for o in out_f], None, None,
                    _ptr(status[1:2]))
            # second problem: h0 = 0, lambda0 = M d_u, u_0 gets -R_inv d_u
            ins_b = ins[:8] + [zeros[:n]]
            _launch("ttc_lqr_rollout", dev, lib.ttc_lqr_rollout, *[_ptr(t) for t in ins_b], _ptr(zeros[:n]),
                    _ptr(M), _ptr(d_u[a:a + n]), 1, n, nh, d, du, T, _F32, *[_ptr(o[a:a + n]) for o in out_b],
                    _ptr(lam0_b[a:a + n]), None, _ptr(status[1:2]))
    st = status.tolist()
    check_fwd_status(st[0])
    if st[1] & _lib.STATUS_TRAJ_NONFINITE:
        raise RuntimeError(TRAJ_NONFINITE_MSG)
    return out_f, out_b, lam0_b


def kkt_grads(A, B, Q, R_inv, lgA, lgB, lgQ, h0, T, fwd, bwd, lam0_b):
    """Gradients of the nine solver inputs from the two problems' trajectories.

    fwd / bwd = (u [N,nh,T,du], states h_1..h_T [N,nh,T,d], costates lambda_1..lambda_T
    [N,nh,T,d]) of the forward problem and of the one driven by r_0 = du; lam0_b its lambda0.
    Per step t (exponent e = t + 1; torch_lqr.py:49-61):
        gA_t = h_t^f lam_{t+1}^b + h_t^b lam_{t+1}^f,   gB_t = lam^b u^f^T + lam^f u^b^T,
        gQ_t = (h^b h^f^T + h^f h^b^T) / 2 (t = T-1: Q_f),   gR_t = u^f u^b,   g_h0 = lambda0^b,
    carried through A_t = 1 + a e^{lgA e}, B_t = B e^{lgB e}, Q_t = D Q D with
    D = e^{lgQ e} (t < T-1), R_t = 1 / R_inv (torch_lqr.py:65-91).  Returns the nine gradients
    (A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0), summed over heads for B and Q."""
    u_f, hs_f, lam_f = fwd
    u_b, hs_b, lam_b = bwd
    N, nh, _, d = hs_f.shape
    du = u_f.shape[-1]
    dt = u_f.dtype
    e = torch.arange(1, T + 1, device=u_f.device, dtype=dt)
    eA = torch.exp(lgA[..., None] * e)                               # [N,nh,T]
    eB = torch.exp(lgB[:, :, None, :] * e[:, None])                  # [N,nh,T,du]
    eQ = torch.exp(lgQ[:, :, None, :] * e[:, None])                  # [N,nh,T,d]
    # gA_t = h_t^f lam^b + h_t^b lam^f with h_t the state before step t (h_0^b = 0)
    gA_t = lam_b * torch.cat([h0[:, :, None], hs_f[:, :, :-1]], dim=2)
    gA_t[:, :, 1:] += hs_b[:, :, :-1] * lam_f[:, :, 1:]
    g_A = (gA_t * eA[..., None]).sum(2)
    g_lgA = ((gA_t * A[:, :, None, :]).sum(-1) * (e * eA)).sum(-1)
    del gA_t
    # grad_B[n] = sum over heads and steps of lam^b (u^f e^lgB)^T + lam^f (u^b e^lgB)^T:
    # one batched GEMM per row with K = heads x steps
    ufe = (u_f * eB).reshape(N, nh * T, du)
    ube = (u_b * eB).reshape(N, nh * T, du)
    lb2 = lam_b.reshape(N, nh * T, d)
    lf2 = lam_f.reshape(N, nh * T, d)
    g_B = lb2.transpose(1, 2) @ ufe + lf2.transpose(1, 2) @ ube
    del ufe, ube
    # B^T lambda per head and step: [N, nh*T, d] @ [N, d, du]
    g_lgB = ((u_f * (lb2 @ B).view(N, nh, T, du) + u_b * (lf2 @ B).view(N, nh, T, du))
             * (e[:, None] * eB)).sum(2)
    del lb2, lf2
    # Q_t = D Q D for t < T-1 (Q_f at T-1): X = h^b D, Y = h^f D over those steps
    X = (hs_b[:, :, :-1] * eQ[:, :, :-1]).reshape(N, nh * (T - 1), d)
    Y = (hs_f[:, :, :-1] * eQ[:, :, :-1]).reshape(N, nh * (T - 1), d)
    S = X.transpose(1, 2) @ Y
    g_Q = 0.5 * (S + S.transpose(-1, -2))
    Qs = Q + Q.transpose(-1, -2)                                      # symmetric
    g_lgQ = (0.5 * (X * (Y @ Qs) + Y * (X @ Qs))).view(N, nh, T - 1, d)
    g_lgQ = (g_lgQ * e[:-1, None]).sum(2)
    del X, Y
    hb, hf = hs_b[:, :, -1], hs_f[:, :, -1]
    g_Qf = 0.5 * (hb[..., :, None] * hf[..., None, :] + hf[..., :, None] * hb[..., None, :])
    g_R = -(u_f * u_b).sum(2) / (R_inv * R_inv)
    return g_A, g_B, g_Q, g_R, g_Qf, g_lgA, g_lgB, g_lgQ, lam0_b


class KKTSolveFunction(torch.autograd.Function):
    """The reference's KKTLQRSolveFunc / kkt_lqr_solve (torch_lqr.py:12-63,120-139) on the
    B200 kernels; same signature as the other solvers (ttc_layer.py:137)."""

    @staticmethod
    def forward(ctx, A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T, save_budget):
        T = int(T)
        N, nh, d, du = _check_shapes(A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T)
        dtype = Q.dtype
        if dtype not in _DTYPES:
            raise TypeError(f"ttc_b200 'kkt' solver supports float32 and bfloat16, got {dtype}")
        inputs = (A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0)
        # The inputs are kept in their own dtype for the backward, which converts one row chunk
        # at a time to fp32: a bf16 layer keeps no full-size fp32 copy between the passes.
        kept = [t.detach().contiguous() for t in inputs]
        args = _prepare(kept, torch.float32)
        dev = Q.device
        u = torch.empty(N, nh, du, device=dev, dtype=torch.float32)
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        lib = _lib.load()
        with torch.cuda.device(dev), torch.profiler.record_function("fwd:ttc_lqr_fwd(kkt)"):
            _launch("ttc_lqr_fwd", dev, lib.ttc_lqr_fwd, *[_ptr(a) for a in args], N, nh, d, du, T,
                    _F32, 0, _ptr(u), None, None, _ptr(status))
        check_fwd_status(int(status.item()))
        del args
        ctx.save_for_backward(*kept)
        ctx.T = T
        ctx.budget = int(save_budget)
        return u.to(dtype)

    @staticmethod
    def backward(ctx, d_u):
        args = ctx.saved_tensors
        T = ctx.T
        d_u = d_u.to(torch.float32).contiguous()
        N, nh, d = args[0].shape
        du = args[1].shape[-1]
        # Rows are independent: the two problems' trajectories and the gradient terms built
        # from them are formed in row chunks of about KKT_WORK_BYTES (beyond that budget: the
        # chunk's fp32 copies of the inputs, and the gradients in the inputs' own dtype).
        rows = max(1, min(N, KKT_WORK_BYTES // (KKT_BYTES_PER_STEP * nh * T * (2 * du + 4 * d))))
        grads = [torch.empty_like(t) for t in args]
        for a in range(0, N, rows):
            sub = [t[a:a + rows].float() for t in args]
            with torch.profiler.record_function("bwd:kkt rollouts"):
                fwd, bwd, lam0_b = _rollouts(sub, T, d_u[a:a + rows], ctx.budget)
            A, B, Q, R, _, lA, lB, lQ, h0 = sub
            for out, g in zip(grads, kkt_grads(A, B, Q, R, lA, lB, lQ, h0, T, fwd, bwd, lam0_b)):
                out[a:a + rows] = g
            del fwd, bwd, lam0_b, sub
        return (*grads, None, None)


def kkt_lqr_solve(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                  save_budget: int | None = None):
    """Drop-in for the reference's ``kkt`` solver (ttc_layer.py:18-22): returns u [N, nh, du]."""
    budget = SAVE_BUDGET_BYTES if save_budget is None else int(save_budget)
    return KKTSolveFunction.apply(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B,
                                  log_gamma_Q, h0, T, budget)
