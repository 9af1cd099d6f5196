"""GPU parity of ``solver_impl="kkt"`` (ttc_b200.kkt: Riccati forward on ttc_lqr_fwd, the
reference's two-problem backward on ttc_lqr_rollout) against the reference's kkt golden
vectors, the oracle, and the fused-convention CUDA backward it must agree with."""
import pytest
import torch

from oracle import ttc_oracle as O
from test_gpu_parity import GRAD_NAMES, SOLVER_CASES, cuda_args, load
from ttc_cases import CONFIGS, layer_weights, solver_inputs_synthetic

pytestmark = pytest.mark.gpu


def _run(solver, args, T, dy, **kw):
    u = solver(*args, T, **kw)
    (u * dy).sum().backward()
    return u.detach(), [a.grad.detach() for a in args]


@pytest.mark.parametrize("case", SOLVER_CASES)
def test_kkt_solver_matches_reference_golden(case):
    from ttc_b200 import kkt_lqr_solve
    z = load(case)
    T = int(z["T"])
    u, grads = _run(kkt_lqr_solve, cuda_args(z), T, torch.from_numpy(z["dy"]).cuda())
    assert O.max_rel(u.cpu(), torch.from_numpy(z["u_kkt"])) < 1e-4
    for gn, g in zip(GRAD_NAMES, grads):
        assert O.max_rel(g.cpu(), torch.from_numpy(z[gn])) < 1e-3, gn


@pytest.mark.parametrize("d,du,nh,N,T", [(16, 16, 16, 64, 64), (32, 32, 8, 6, 96), (32, 16, 5, 7, 33),
                                        (64, 64, 2, 3, 20)])
def test_kkt_agrees_with_fused_backward(d, du, nh, N, T):
    """Same semantics, different algorithm: the kkt gradients equal the adjoint kernel's."""
    from ttc_b200 import cuda_lqr_solve, kkt_lqr_solve
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(N, nh, d, du, seed=70 + d)]
    dy = torch.randn(N, nh, du, device="cuda", generator=torch.Generator(device="cuda").manual_seed(d))
    mk = lambda: [a.to("cuda", torch.float32).requires_grad_(True) for a in host]  # noqa: E731
    u_k, g_k = _run(kkt_lqr_solve, mk(), T, dy)
    u_c, g_c = _run(cuda_lqr_solve, mk(), T, dy)
    assert O.max_rel(u_k, u_c) < 1e-6  # the same forward kernel (without / with M saved)
    for name, a, b in zip(GRAD_NAMES, g_k, g_c):
        assert O.max_rel(a, b) < 1e-4, name


def test_kkt_row_chunks_give_the_same_gradients():
    from ttc_b200 import kkt_lqr_solve
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(9, 4, 16, 16, seed=71)]
    dy = torch.randn(9, 4, 16, device="cuda")
    mk = lambda: [a.to("cuda", torch.float32).requires_grad_(True) for a in host]  # noqa: E731
    _, whole = _run(kkt_lqr_solve, mk(), 24, dy)
    _, chunked = _run(kkt_lqr_solve, mk(), 24, dy, save_budget=2 * 4 * 16 * 16 * 4)
    for a, b in zip(whole, chunked):
        assert torch.equal(a, b)


@pytest.mark.parametrize("case", ["layer_cfg1", "layer_cfg2"])
def test_kkt_layer_matches_reference_golden(case):
    """TTCLayer(solver_impl="kkt") against the reference layer (its kkt gradients)."""
    from ttc_b200 import TTCLayer
    z = load(case)
    cfg = CONFIGS[int(z["cfg"])]
    layer = TTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank, solver_impl="kkt")
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    layer = layer.cuda()
    x = torch.from_numpy(z["x"]).cuda()[None].requires_grad_(True)
    y = layer(x, T=int(z["T"]))
    assert O.max_rel(y[0].detach().cpu(), torch.from_numpy(z["y"])) < 1e-4
    if "g_x" not in z:
        return
    (y[0] * torch.from_numpy(z["dy"]).cuda()).sum().backward()
    assert O.max_rel(x.grad[0].cpu(), torch.from_numpy(z["g_x"])) < 1e-3
    for pn, p in layer.named_parameters():
        s = int(z["stride_" + pn])
        assert O.max_rel(p.grad[::s].cpu(), torch.from_numpy(z["g_" + pn])) < 1e-3, pn


def test_kkt_bf16_inputs_run_in_fp32():
    """bf16 activations: state and gradient math in fp32 (the reference's kkt is fp32 only),
    outputs cast back; agrees with the fp32 solve on the same bf16-rounded inputs."""
    from ttc_b200 import kkt_lqr_solve
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(6, 4, 32, 32, seed=72)]
    dy = torch.randn(6, 4, 32, device="cuda")
    a16 = [a.to("cuda", torch.bfloat16).requires_grad_(True) for a in host]
    a32 = [a.to("cuda", torch.bfloat16).float().requires_grad_(True) for a in host]
    u16, g16 = _run(kkt_lqr_solve, a16, 32, dy.bfloat16())
    u32, g32 = _run(kkt_lqr_solve, a32, 32, dy.bfloat16().float())
    assert u16.dtype == torch.bfloat16 and all(g.dtype == torch.bfloat16 for g in g16)
    assert O.max_rel(u16.float(), u32) < 1e-2
    for name, a, b in zip(GRAD_NAMES, g16, g32):
        assert O.max_rel(a.float(), b) < 1e-2, name


def test_kkt_backward_row_chunks(monkeypatch):
    """A small work budget splits the backward's trajectories into row chunks: same gradients."""
    import ttc_b200.kkt as K
    from ttc_b200 import kkt_lqr_solve
    host = [torch.from_numpy(a) for a in solver_inputs_synthetic(10, 4, 16, 16, seed=73)]
    dy = torch.randn(10, 4, 16, device="cuda")
    mk = lambda: [a.to("cuda", torch.float32).requires_grad_(True) for a in host]  # noqa: E731
    _, whole = _run(kkt_lqr_solve, mk(), 24, dy)
    monkeypatch.setattr(K, "KKT_WORK_BYTES", 3 * K.KKT_BYTES_PER_STEP * 4 * 24 * (2 * 16 + 4 * 16))
    _, chunked = _run(kkt_lqr_solve, mk(), 24, dy)
    for name, a, b in zip(GRAD_NAMES, chunked, whole):
        assert O.max_rel(a, b) < 1e-6, name
