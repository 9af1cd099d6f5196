"""GPU parity of the solve with Q_f given as the layer's rank-r mixture
(ttc_lqr_fwd_mix / ttc_lqr_bwd_mix: Q_f = sum_r coeff_Qf[..., r] Q_basis[r] formed inside the
kernels, ttc_layer.py:119-123) against the same solve with Q_f materialised by einsum and
passed to ttc_lqr_fwd / ttc_lqr_bwd: u, and the gradients of every input (coeff_Qf and
Q_basis through the einsum's autograd on the materialised side)."""
import pytest
import torch

from ttc_cases import solver_inputs_synthetic

pytestmark = pytest.mark.gpu


def _inputs(N, nh, d, rQ, dtype, seed):
    A, B, Q, R, Qf, lA, lB, lQ, h0 = [torch.from_numpy(a).cuda() for a in
                                      solver_inputs_synthetic(N, nh, d, d, seed)]
    g = torch.Generator(device="cuda").manual_seed(seed + 11)
    coeff = torch.nn.functional.normalize(torch.rand(N, nh, rQ, device="cuda", generator=g), dim=-1)
    G = torch.randn(rQ, d, d, device="cuda", generator=g) * 0.3
    basis = G @ G.transpose(1, 2) / d ** 0.5
    return [t.to(dtype) for t in (A, B, Q, R, coeff, basis, lA, lB, lQ, h0)]


def _maxrel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


CASES = [(256, 16, 16, 16, 64), (100, 12, 16, 16, 5), (64, 32, 32, 32, 16), (37, 24, 32, 32, 9),
         (50, 16, 16, 8, 7)]


@pytest.mark.parametrize("dtype,tol_u,tol_g", [(torch.float32, 1e-5, 1e-4), (torch.bfloat16, 2e-2, 5e-2)])
@pytest.mark.parametrize("case", CASES)
def test_mixed_qf_matches_materialised(case, dtype, tol_u, tol_g):
    from ttc_b200.solver import LQRSolveFunction, LQRSolveMixFunction, SAVE_BUDGET_BYTES, mix_available
    N, nh, d, rQ, T = case
    assert mix_available(N, nh, d, d, rQ, dtype)
    xs = _inputs(N, nh, d, rQ, dtype, seed=N + nh)
    xa = [t.clone().requires_grad_(True) for t in xs]
    xb = [t.clone().requires_grad_(True) for t in xs]
    ua, _ = LQRSolveMixFunction.apply(*xa, T)
    A, B, Q, R, coeff, basis, lA, lB, lQ, h0 = xb
    Qf = torch.einsum("...r,rmn->...mn", coeff, basis)
    ub, _ = LQRSolveFunction.apply(A, B, Q, R, Qf, lA, lB, lQ, h0, T, SAVE_BUDGET_BYTES)
    assert _maxrel(ua, ub) <= tol_u
    g = torch.Generator(device="cuda").manual_seed(3)
    du = torch.randn(ua.shape, device="cuda", generator=g).to(dtype)
    ua.backward(du)
    ub.backward(du)
    names = ["A_diag", "B", "Q", "R_inv", "coeff_Qf", "Q_basis", "lgA", "lgB", "lgQ", "h0"]
    for n, a, b in zip(names, xa, xb):
        assert a.grad is not None and a.grad.dtype == a.dtype, n
        assert _maxrel(a.grad, b.grad) <= tol_g, f"{n}: {_maxrel(a.grad, b.grad):.2e}"


def test_mixed_qf_deterministic():
    from ttc_b200.solver import LQRSolveMixFunction
    xs = _inputs(300, 16, 16, 16, torch.float32, seed=5)
    outs = []
    for _ in range(2):
        x = [t.clone().requires_grad_(True) for t in xs]
        u, _ = LQRSolveMixFunction.apply(*x, 12)
        u.backward(torch.ones_like(u))
        outs.append([u.detach()] + [t.grad for t in x])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_mix_not_offered_where_unsupported():
    from ttc_b200.solver import mix_available
    assert not mix_available(64, 8, 64, 64, 64, torch.float32)   # d = 64: CUDA-core backward
    assert not mix_available(8, 16, 16, 16, 16, torch.float32, save_budget=0)  # M not kept
    assert not mix_available(8, 100, 16, 16, 16, torch.float32)  # more than 64 heads
    assert not mix_available(8, 32, 32, 32, 64, torch.float32)   # basis too large for the forward
