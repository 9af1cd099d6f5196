"""The layer's low-rank solve (ttc_lqr_fwd_lowrank / ttc_lqr_bwd_lowrank: B, Q and Q_f mixed
inside the solver kernels) against the same solve with B and Q formed first by the
einsums of ttc/layers/ttc_layer.py:115-118 (lowrank_mix, cuBLAS) and Q_f mixed in the kernels
(ttc_lqr_fwd_mix / ttc_lqr_bwd_mix), and the epilogue's row l2norm kernel against the fla
formula (fla/modules/l2norm.py:42) and its autograd.  Gradients are compared for every
coefficient and basis, through autograd of the einsums on the reference side."""
import pytest
import torch

from oracle import ttc_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def cuda_lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import build as ttc_build
    ttc_build.build()
    from ttc_b200 import _lib
    return _lib.load()


def _parts(N, nh, d, rB, rQ, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)

    def rn(*s):
        return torch.randn(*s, device="cuda", generator=g)

    A = torch.nn.functional.normalize(torch.rand(N, nh, d, device="cuda", generator=g), dim=-1)
    cB = torch.nn.functional.normalize(rn(N, rB), dim=-1)
    Bb = rn(rB, d, d) * 0.3
    cQ = torch.nn.functional.normalize(torch.rand(N, rQ, device="cuda", generator=g), dim=-1)
    G = rn(rQ, d, d) * 0.3
    Qb = G @ G.transpose(1, 2) / d ** 0.5
    R = torch.nn.functional.softplus(torch.rand(N, nh, d, device="cuda", generator=g))
    cQf = torch.nn.functional.normalize(torch.rand(N, nh, rQ, device="cuda", generator=g), dim=-1)
    lgA = -torch.nn.functional.softplus(rn(N, nh)) - 1.3
    lgB = -torch.nn.functional.softplus(rn(N, nh, d)) - 1.3
    lgQ = -torch.nn.functional.softplus(rn(N, nh, d)) - 1.3
    h0 = rn(N, nh, d)
    parts = [A, cB, Bb, cQ, Qb, R, cQf, lgA, lgB, lgQ, h0]
    return [p.to(dtype).contiguous().requires_grad_(True) for p in parts]


@pytest.mark.parametrize("d,nh,N,rB,rQ,T", [(16, 16, 40, 16, 16, 24), (16, 5, 9, 8, 12, 7),
                                             (32, 32, 12, 32, 32, 20), (32, 12, 7, 16, 24, 9)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_lowrank_solve_matches_mixed_then_solved(d, nh, N, rB, rQ, T, dtype):
    from ttc_b200.reductions import lowrank_mix
    from ttc_b200.solver import LQRSolveLowRankFunction, LQRSolveMixFunction, mix_available
    assert mix_available(N, nh, d, d, rQ, dtype)
    parts = _parts(N, nh, d, rB, rQ, dtype, seed=d + nh + N)
    ref_parts = [p.detach().clone().requires_grad_(True) for p in parts]
    dy = torch.randn(N, nh, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3)).to(dtype)

    u, st = LQRSolveLowRankFunction.apply(*parts, T)
    (u.float() * dy.float()).sum().backward()

    A, cB, Bb, cQ, Qb, R, cQf, lgA, lgB, lgQ, h0 = ref_parts
    B = lowrank_mix(cB, Bb)
    Q = lowrank_mix(cQ, Qb)
    u_ref, st_ref = LQRSolveMixFunction.apply(A, B, Q, R, cQf, Qb, lgA, lgB, lgQ, h0, T)
    (u_ref.float() * dy.float()).sum().backward()
    assert int(st) == 0 and int(st_ref) == 0
    # fp32: the mixtures differ from cuBLAS's only in summation order; bf16: both round the
    # mixtures to bf16, so an element can land one bf16 step apart
    fwd_tol, grad_tol = (1e-5, 1e-4) if dtype == torch.float32 else (2e-2, 5e-2)
    assert O.max_rel(u.detach().float().cpu(), u_ref.detach().float().cpu()) < fwd_tol
    names = ["A_diag", "coeff_B", "B_basis", "coeff_Q", "Q_basis", "R_inv", "coeff_Qf", "lgA", "lgB", "lgQ", "h0"]
    for name, p, q in zip(names, parts, ref_parts):
        assert p.grad is not None and p.grad.dtype == p.dtype, name
        assert O.max_rel(p.grad.float().cpu(), q.grad.float().cpu()) < grad_tol, name


def test_lowrank_forward_without_grad_keeps_no_state():
    from ttc_b200.solver import LQRSolveLowRankFunction
    parts = [p.detach() for p in _parts(6, 4, 16, 8, 8, torch.float32, seed=1)]
    with torch.no_grad():
        u, st = LQRSolveLowRankFunction.apply(*parts, 10)
    g = [p.requires_grad_(True) for p in _parts(6, 4, 16, 8, 8, torch.float32, seed=1)]
    u2, _ = LQRSolveLowRankFunction.apply(*g, 10)
    assert torch.equal(u, u2.detach())


@pytest.mark.parametrize("n", [16, 32, 64, 7, 48])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_rownorm_matches_formula(n, dtype):
    from ttc_b200.epilogue import rownorm
    g = torch.Generator(device="cuda").manual_seed(n)
    x = (torch.randn(37, 5, n, device="cuda", generator=g) * 1e-3).to(dtype)
    gy = torch.randn(37, 5, n, device="cuda", generator=g).to(dtype)
    xa = x.clone().requires_grad_(True)
    y = rownorm(xa)
    y.backward(gy)
    xr = x.clone().requires_grad_(True)
    xf = xr.float()
    yr = (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)).to(dtype)
    yr.backward(gy)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert y.dtype == dtype and xa.grad.dtype == dtype
    assert O.max_rel(y.float().cpu(), yr.detach().float().cpu()) < tol
    assert O.max_rel(xa.grad.float().cpu(), xr.grad.float().cpu()) < (1e-5 if dtype == torch.float32 else 2e-2)
