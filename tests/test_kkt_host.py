"""The GPU kkt solver's gradient assembly (ttc_b200.kkt.kkt_grads: the reference's kkt outer
products, torch_lqr.py:49-61, carried through the time-varying system in closed form) on the
CPU, fed with the oracle's trajectories, against autograd through the oracle's kkt solver."""
import pytest
import torch

from oracle import ttc_oracle as O
from ttc_cases import solver_inputs_synthetic

NAMES = ["A_diag", "B", "Q", "R_inv", "Q_f", "lgA", "lgB", "lgQ", "h0"]


@pytest.mark.parametrize("N,nh,d,du,T,seed,sym", [(3, 2, 16, 16, 12, 1, True), (2, 3, 32, 16, 7, 2, False),
                                                 (2, 2, 16, 16, 1, 3, False), (2, 2, 16, 16, 2, 4, True)])
def test_kkt_grads_match_oracle_autograd(N, nh, d, du, T, seed, sym):
    from ttc_b200.kkt import kkt_grads
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(N, nh, d, du, seed)]
    g = torch.Generator().manual_seed(seed)
    if not sym:  # the closed form keeps the non-symmetric part of Q where it enters
        host[2] = host[2] + 0.3 * torch.randn(N, d, d, generator=g, dtype=torch.float64)
    leaves = [a.clone().requires_grad_(True) for a in host]
    u = O.kkt_solve(*leaves, T)
    dy = torch.randn(u.shape, generator=g, dtype=torch.float64)
    (u * dy).sum().backward()
    A, B, Q, R, _, lA, lB, lQ, h0 = host
    uf, hf, lf, _, _ = O.fused_trajectory(*host, T)
    ub, hb, lb, l0b, _ = O.fused_trajectory(*host[:8], torch.zeros_like(h0), T, r0=dy)
    got = kkt_grads(A, B, Q, R, lA, lB, lQ, h0, T, (uf, hf, lf), (ub, hb, lb), l0b)
    # the oracle's kkt solves its gain systems in fp32, as the reference (lin_solver_lqr.py:175-177)
    for name, a, leaf in zip(NAMES, got, leaves):
        assert O.max_rel(a, leaf.grad) < 1e-6, name
