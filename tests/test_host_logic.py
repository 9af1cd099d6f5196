"""CPU tests of the host-side mirror of the reference interface (no GPU needed).

The product layer (ttc_b200.TTCLayer) runs its elementwise prologue as a CUDA kernel and
the LQR solve in the CUDA library; here its remaining host code (einsums, gamma bias,
epilogue, shapes) is exercised on the CPU with the PyTorch prologue of prologue_ref.py and
the oracle's solver put in their places, and compared with the reference's golden layer
outputs.  The GPU tests cover the kernels themselves."""
import os

import numpy as np
import pytest
import torch

from oracle import ttc_oracle as O
from prologue_ref import _l2norm, prologue_torch
from ttc_cases import CONFIGS, layer_weights

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture
def cpu_prologue(monkeypatch):
    """Swap the layer's CUDA prologue and epilogue for PyTorch ones (test-only)."""
    import ttc_b200.layer as L
    monkeypatch.setattr(L, "prologue", prologue_torch)
    monkeypatch.setattr(L, "rownorm", _l2norm)


def test_product_layer_has_no_cpu_path():
    """Without the stand-ins the product layer refuses CPU tensors instead of falling back."""
    from ttc_b200 import TTCLayer
    layer = TTCLayer(8, 6, 16, 2, 16, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.randn(1, 3, 8), T=2)


def test_registry_and_unknown_solver():
    from ttc_b200 import LQR_SOLVER_IMPL_MAP, TTCLayer, cuda_lqr_solve
    assert LQR_SOLVER_IMPL_MAP["cuda"] is cuda_lqr_solve
    assert LQR_SOLVER_IMPL_MAP["fused"] is cuda_lqr_solve
    with pytest.raises(AssertionError, match="Unknown LQR solver"):
        TTCLayer(8, 8, 16, 2, 16, 16, solver_impl="triton")


@pytest.mark.parametrize("kw", [{}, {"bias": True}, {"gamma_bias": True}, {"u_dim": 8},
                                {"q_reparam": "cholesky"}])
def test_parameters_match_reference_layout(kw):
    """Same parameter names and shapes as ttc/layers/ttc_layer.py:56-68, so a reference
    state_dict loads 1:1."""
    from ttc_b200 import TTCLayer
    a = TTCLayer(32, 24, 16, 4, 8, 16, **kw)
    b = O.TTCLayerOracle(32, 24, 16, 4, 8, 16, **kw)
    sa, sb = a.state_dict(), b.state_dict()
    assert list(sa) == list(sb)
    assert all(sa[k].shape == sb[k].shape for k in sa)
    a.load_state_dict(sb)


def test_init_distributions():
    from ttc_b200 import TTCLayer
    torch.manual_seed(0)
    layer = TTCLayer(32, 32, 16, 8, 16, 16, gamma_bias=True)
    assert torch.allclose(layer.Qs, layer.Qs.transpose(1, 2))
    assert (torch.linalg.eigvalsh(layer.Qs.double()) > -1e-12).all()
    assert abs(layer.Bs.std().item() - 0.02) < 0.002
    assert torch.allclose(layer.bias_gamma, torch.full_like(layer.bias_gamma, -np.log(4.0)))


def test_zero_horizon_returns_zeros():
    from ttc_b200 import TTCLayer
    layer = TTCLayer(32, 24, 16, 4, 16, 16)
    y = layer(torch.randn(2, 3, 32), T=0)
    assert y.shape == (2, 3, 24) and not y.any()


def test_cuda_solver_rejects_cpu_tensors():
    from ttc_b200 import cuda_lqr_solve
    from ttc_cases import solver_inputs_synthetic
    host = [torch.from_numpy(a).float() for a in solver_inputs_synthetic(2, 2, 16, 16, seed=1)]
    with pytest.raises(ValueError, match="CUDA tensors"):
        cuda_lqr_solve(*host, 4)


def test_registry_has_gpu_kkt():
    """The reference's "kkt" name maps to the GPU kkt solver; "riccati" stays the CPU oracle."""
    from ttc_b200 import LQR_SOLVER_IMPL_MAP, kkt_lqr_solve
    assert LQR_SOLVER_IMPL_MAP["kkt"] is kkt_lqr_solve
    assert "riccati" not in LQR_SOLVER_IMPL_MAP


def test_trajectory_host_checks():
    """lqr_trajectory validates before any launch: a per-step cost passed as r0 points to
    r_traj, wrong r0 / r_traj shapes and both at once are errors, and CPU tensors have no
    path."""
    from ttc_b200 import kkt_lqr_solve, lqr_trajectory
    from ttc_cases import solver_inputs_synthetic
    host = [torch.from_numpy(a).float() for a in solver_inputs_synthetic(2, 2, 16, 16, seed=1)]
    with pytest.raises(AssertionError, match="every step goes in r_traj"):
        lqr_trajectory(*host, 4, r0=torch.zeros(2, 2, 4, 16))
    with pytest.raises(AssertionError, match="r0 must be"):
        lqr_trajectory(*host, 4, r0=torch.zeros(2, 16))
    with pytest.raises(AssertionError, match="r_traj must be"):
        lqr_trajectory(*host, 4, r_traj=torch.zeros(2, 2, 5, 16))
    with pytest.raises(ValueError, match="not both"):
        lqr_trajectory(*host, 4, r0=torch.zeros(2, 2, 16), r_traj=torch.zeros(2, 2, 4, 16))
    with pytest.raises(ValueError, match="CUDA tensors"):
        lqr_trajectory(*host, 4, r_traj=torch.zeros(2, 2, 4, 16))
    with pytest.raises(ValueError, match="CUDA tensors"):
        lqr_trajectory(*host, 4)
    with pytest.raises(ValueError, match="CUDA tensors"):
        kkt_lqr_solve(*host, 4)


def test_solver_shape_contract():
    from ttc_b200 import cuda_lqr_solve
    from ttc_cases import solver_inputs_synthetic
    host = [torch.from_numpy(a).float() for a in solver_inputs_synthetic(2, 2, 16, 16, seed=1)]
    host[2] = host[2][:, :8]
    with pytest.raises(AssertionError, match="Q must be"):
        cuda_lqr_solve(*host, 4)


@pytest.mark.parametrize("case", ["layer_cfg2", "layer_cfg3"])
def test_product_prologue_epilogue_against_reference(case, cpu_prologue):
    """ttc_b200.TTCLayer's own prologue/epilogue code with the oracle fused solver in the
    solver slot reproduces the reference layer's y and gradients."""
    from ttc_b200 import TTCLayer
    z = np.load(os.path.join(GOLDEN, case + ".npz"))
    cfg = CONFIGS[int(z["cfg"])]
    layer = TTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    layer.solver = O.fused_solve
    x = torch.from_numpy(z["x"])[None].requires_grad_(True)
    y = layer(x, T=int(z["T"]))
    assert O.max_rel(y[0], torch.from_numpy(z["y"])) < 1e-4
    (y[0] * torch.from_numpy(z["dy"])).sum().backward()
    assert O.max_rel(x.grad[0], torch.from_numpy(z["g_x"])) < 1e-3
    for pn, p in layer.named_parameters():
        s = int(z["stride_" + pn])
        assert O.max_rel(p.grad[::s], torch.from_numpy(z["g_" + pn])) < 1e-3, pn


def test_four_dim_input_convention(cpu_prologue):
    from ttc_b200 import TTCLayer
    layer = TTCLayer(8, 6, 16, 3, 16, 16)
    layer.solver = O.fused_solve
    x = torch.randn(2, 2, 3, 8)
    y4 = layer(x, T=4)
    y3 = layer(x.reshape(2, 6, 8), T=4).reshape(2, 2, 3, 6)
    assert y4.shape == (2, 2, 3, 6)
    assert torch.equal(y4, y3)


@pytest.mark.parametrize("K", [4096, 300])
def test_chunked_weight_gradients_match_torch(K):
    """ttc_b200.reductions: linear / lowrank_mix give F.linear / einsum values and gradients
    (K-chunked batched weight-gradient GEMM when K splits, a plain GEMM otherwise)."""
    import torch.nn.functional as F
    from ttc_b200.reductions import _chunks, linear, lowrank_mix
    assert (_chunks(K) > 1) == (K == 4096)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(K, 12, dtype=torch.float64, generator=g)
    w = torch.randn(7, 12, dtype=torch.float64, generator=g)
    b = torch.randn(7, dtype=torch.float64, generator=g)
    gy = torch.randn(K, 7, dtype=torch.float64, generator=g)
    ins = [t.clone().requires_grad_(True) for t in (x, w, b)]
    ref = [t.clone().requires_grad_(True) for t in (x, w, b)]
    linear(*ins).backward(gy)
    F.linear(*ref).backward(gy)
    for a, r in zip(ins, ref):
        assert torch.allclose(a.grad, r.grad, rtol=1e-12, atol=1e-10)
    c = torch.randn(K // 4, 4, 5, dtype=torch.float64, generator=g)
    basis = torch.randn(5, 3, 6, dtype=torch.float64, generator=g)
    go = torch.randn(K // 4, 4, 3, 6, dtype=torch.float64, generator=g)
    a1, a2 = c.clone().requires_grad_(True), basis.clone().requires_grad_(True)
    r1, r2 = c.clone().requires_grad_(True), basis.clone().requires_grad_(True)
    out = lowrank_mix(a1, a2)
    assert torch.allclose(out, torch.einsum("...r,rmn->...mn", c, basis), rtol=1e-12)
    out.backward(go)
    torch.einsum("...r,rmn->...mn", r1, r2).backward(go)
    assert torch.allclose(a1.grad, r1.grad, rtol=1e-12, atol=1e-10)
    assert torch.allclose(a2.grad, r2.grad, rtol=1e-12, atol=1e-10)


def test_bf16_values_are_exact_tf32_operands():
    """The kernels skip the A_hi * B_lo terms of their 3xTF32 products for bf16 activations:
    B and Q then hold bf16 values (the solver's inputs, or the layer's mixtures rounded to
    bf16), and a bf16 value widened to fp32 has its low 16 mantissa bits zero, so the tf32
    truncation the tensor cores apply (the low 13 bits) leaves it unchanged and its residual
    B_lo is exactly zero.  Checked over every finite bf16 bit pattern."""
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    f = bits.float()
    f = f[torch.isfinite(f)]
    u = f.view(torch.int32)
    assert torch.equal(u & 0x1FFF, torch.zeros_like(u))
    hi = (u & ~0x1FFF).view(torch.float32)
    assert torch.equal(f - hi, torch.zeros_like(f))
