"""Pin the CPU oracle to the reference: every oracle function against the golden vectors
that tests/golden/make_golden.py produced by running the reference package itself."""
import os

import numpy as np
import pytest
import torch

from oracle import ttc_oracle as O
from ttc_cases import CONFIGS, SOLVER_ARG_NAMES, layer_weights

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SOLVER_CASES = ["solver_bench_d16", "solver_synth_d32", "solver_synth_d64", "solver_T1",
                "solver_T2", "solver_growth", "prologue_cfg1", "prologue_cfg2", "prologue_cfg3",
                "prologue_cfg4"]
FAST_CASES = [c for c in SOLVER_CASES if c not in ("solver_synth_d64", "prologue_cfg4")]
GRAD_NAMES = ["g_" + n for n in SOLVER_ARG_NAMES]


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def solver_args(z, dtype=torch.float32):
    return [torch.from_numpy(z[n]).to(dtype) for n in SOLVER_ARG_NAMES]


@pytest.mark.parametrize("case", SOLVER_CASES)
def test_riccati_matches_reference(case):
    z = load(case)
    u = O.riccati_solve(*solver_args(z), int(z["T"]))
    assert O.max_rel(u, torch.from_numpy(z["u_riccati"])) < 1e-4


@pytest.mark.parametrize("case", FAST_CASES)
def test_kkt_matches_reference(case):
    z = load(case)
    leaves = [a.requires_grad_(True) for a in solver_args(z)]
    u = O.kkt_solve(*leaves, int(z["T"]))
    assert O.max_rel(u, torch.from_numpy(z["u_kkt"])) < 1e-4
    (u * torch.from_numpy(z["dy"])).sum().backward()
    for gn, leaf in zip(GRAD_NAMES, leaves):
        assert O.max_rel(leaf.grad, torch.from_numpy(z[gn])) < 2e-3, gn


@pytest.mark.parametrize("case", SOLVER_CASES)
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_fused_restatement_matches_reference(case, dtype):
    """The fused (symplectic) restatement against the reference's riccati forward and kkt
    gradients (same symmetric Q/Q_f convention as the reference fused backward)."""
    z = load(case)
    leaves = [a.requires_grad_(True) for a in solver_args(z, dtype)]
    u = O.fused_solve(*leaves, int(z["T"]))
    tol_u = 1e-4
    assert O.max_rel(u, torch.from_numpy(z["u_riccati"])) < tol_u
    (u * torch.from_numpy(z["dy"]).to(dtype)).sum().backward()
    for gn, leaf in zip(GRAD_NAMES, leaves):
        assert O.max_rel(leaf.grad, torch.from_numpy(z[gn])) < 1e-3, gn


def test_riccati_bf16_matches_reference():
    z = load("prologue_cfg3_bf16")
    u = O.riccati_solve(*solver_args(z, torch.bfloat16), int(z["T"]))
    assert O.max_rel(u.float(), torch.from_numpy(z["u_riccati"])) < 2e-2


def _oracle_layer(cfg, solver, dtype=torch.float32):
    layer = O.TTCLayerOracle(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                             solver_impl=solver)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    return layer.to(dtype)


@pytest.mark.parametrize("case,solver", [("layer_cfg1", "riccati"), ("layer_cfg2", "kkt"),
                                         ("layer_cfg2", "fused"), ("layer_cfg3", "fused"),
                                         ("layer_cfg5", "fused")])
def test_layer_matches_reference(case, solver):
    z = load(case)
    cfg = CONFIGS[int(z["cfg"])]
    layer = _oracle_layer(cfg, solver)
    x = torch.from_numpy(z["x"])[None].requires_grad_("g_x" in z)
    y = layer(x, T=int(z["T"]))
    assert O.max_rel(y[0], torch.from_numpy(z["y"])) < 1e-4
    if "g_x" not in z:
        return
    (y[0] * torch.from_numpy(z["dy"])).sum().backward()
    assert O.max_rel(x.grad[0], torch.from_numpy(z["g_x"])) < 1e-3
    for pn, p in layer.named_parameters():
        s = int(z["stride_" + pn])
        assert O.max_rel(p.grad[::s], torch.from_numpy(z["g_" + pn])) < 1e-3, pn


def test_layer_bf16_matches_reference():
    z = load("layer_cfg3_bf16")
    cfg = CONFIGS[int(z["cfg"])]
    layer = _oracle_layer(cfg, "riccati", torch.bfloat16)
    y = layer(torch.from_numpy(z["x"]).to(torch.bfloat16)[None], T=int(z["T"]))
    assert O.max_rel(y[0].float(), torch.from_numpy(z["y"])) < 2e-2


@pytest.mark.parametrize("cid", [3, 5])
def test_layer_bf16_rounded_oracle_matches_reference(cid):
    """The bf16 oracle of configs 3 and 5: the fp32 layer on bf16-rounded x, dy and weights
    (reference kkt gradients in the fixture), and the reference's own bf16 forward within the
    bf16 bar of it."""
    z = load(f"layer_cfg{cid}_bf16grad")
    cfg = CONFIGS[cid]
    layer = O.TTCLayerOracle(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank,
                             solver_impl="fused")
    layer.load_state_dict({k: torch.from_numpy(v).to(torch.bfloat16).float()
                           for k, v in layer_weights(cfg).items()})
    x = torch.from_numpy(z["x"]).to(torch.bfloat16).float()[None].requires_grad_(True)
    y = layer(x, T=int(z["T"]))
    assert O.max_rel(y[0], torch.from_numpy(z["y"])) < 1e-4
    assert O.max_rel(torch.from_numpy(z["y_refbf16"]), torch.from_numpy(z["y"])) < 2e-2
    (y[0] * torch.from_numpy(z["dy"]).to(torch.bfloat16).float()).sum().backward()
    assert O.max_rel(x.grad[0], torch.from_numpy(z["g_x"])) < 1e-3
    for pn, p in layer.named_parameters():
        s = int(z["stride_" + pn])
        assert O.max_rel(p.grad[::s], torch.from_numpy(z["g_" + pn])) < 1e-3, pn


def test_kkt_fp64_against_riccati_autograd():
    """Cross-solver agreement the reference's own bench relies on: the kkt adjoint equals
    autograd through the riccati sweep (Q/Q_f compared on their symmetric parts)."""
    z = load("solver_bench_d16")
    a1 = [a.requires_grad_(True) for a in solver_args(z, torch.float64)]
    a2 = [a.detach().clone().requires_grad_(True) for a in a1]
    T = int(z["T"])
    dy = torch.from_numpy(z["dy"]).double()
    (O.riccati_solve(*a1, T, solve_dtype=None) * dy).sum().backward()
    (O.kkt_solve(*a2, T) * dy).sum().backward()
    sym = lambda g: (g + g.transpose(-1, -2)) / 2
    for i, (p, q) in enumerate(zip(a1, a2)):
        g1, g2 = p.grad, q.grad
        if i in (2, 4):
            g1, g2 = sym(g1), sym(g2)
        assert O.max_rel(g2, g1) < 1e-5, SOLVER_ARG_NAMES[i]
