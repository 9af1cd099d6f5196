"""Parity with the reference's own GPU solver, the Triton ``fused`` path
(ttc/solvers/fused_lqr.py:255-304), the north star's gradient target.

The fixtures ``tests/golden/fused_*.npz`` were written by ``tests/golden/make_fused_golden.py``,
which ran the unmodified reference package on a B200: the fused solver's u and nine gradients
on the inputs and upstream gradient of every solver fixture, on solver inputs captured from
the reference layer prologue at the geometry of configs 3 and 5, and
``TTCLayer(solver_impl="fused")`` forward + backward for configs 3 and 5 (fp32, and bf16
activations for config 5).  Tolerances (max-rel = max|out - ref| / max|ref|): u / y 1e-4 in
fp32, gradients 1e-3 in fp32; bf16 activations 2e-2 for y and 5e-2 for the gradients.
"""
import os

import numpy as np
import pytest
import torch

from oracle import ttc_oracle as O
from ttc_cases import CONFIGS, SOLVER_ARG_NAMES, layer_weights

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GRAD_NAMES = ["g_" + n for n in SOLVER_ARG_NAMES]
FWD_TOL_F32, GRAD_TOL_F32, FWD_TOL_BF16, GRAD_TOL_BF16 = 1e-4, 1e-3, 2e-2, 5e-2

# the solver fixtures of make_golden.py (their inputs and upstream gradients), and inputs
# captured from the reference prologue at configs 3 and 5 (2 rows, all 32 heads)
SOLVER_CASES = ["solver_bench_d16", "solver_synth_d32", "solver_synth_d64", "solver_T1",
                "solver_T2", "solver_growth", "prologue_cfg1", "prologue_cfg2", "prologue_cfg4",
                "capture_cfg3", "capture_cfg5"]


@pytest.fixture(scope="module", autouse=True)
def cuda_lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import build as ttc_build
    ttc_build.build()
    from ttc_b200 import _lib
    return _lib.load()


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def _spread(case, z):
    """How far the reference's fused solver is from the reference's own riccati u and kkt
    gradients on this case (0 where make_golden.py has no riccati / kkt fixture).  On two
    cases the fused solver itself departs from them beyond the tolerances: the growth case
    (state growth ~3e5 over the horizon: 1.2e-4 in u, 2.3e-3 in the gradients) and the
    config-4 geometry (d = 64, T = 512: 8.4e-4 in u, 2.5e-3 in the gradients).  The CUDA path
    stays within the tolerances of riccati / kkt there (tests/test_gpu_parity.py), so against
    fused it is held to the tolerance plus that spread."""
    path = os.path.join(GOLDEN, case + ".npz")
    if not os.path.exists(path):
        return 0.0, {n: 0.0 for n in GRAD_NAMES}
    g = load(case)
    u = O.max_rel(torch.from_numpy(z["u_fused"]), torch.from_numpy(g["u_riccati"]))
    return u, {n: O.max_rel(torch.from_numpy(z[n]), torch.from_numpy(g[n])) for n in GRAD_NAMES}


@pytest.mark.parametrize("case", SOLVER_CASES)
@pytest.mark.parametrize("save_budget", [None, 0], ids=["saved", "recompute"])
def test_solver_matches_reference_fused(case, save_budget):
    from ttc_b200 import cuda_lqr_solve
    z = load("fused_" + case)
    T = int(z["T"])
    spread_u, spread_g = _spread(case, z)
    args = [torch.from_numpy(z[n]).to("cuda", torch.float32).requires_grad_(True) for n in SOLVER_ARG_NAMES]
    u = cuda_lqr_solve(*args, T, save_budget=save_budget)
    (u * torch.from_numpy(z["dy"]).cuda()).sum().backward()
    errs = {"u": O.max_rel(u.detach().cpu(), torch.from_numpy(z["u_fused"]))}
    for gname, a in zip(GRAD_NAMES, args):
        errs[gname] = O.max_rel(a.grad.cpu(), torch.from_numpy(z[gname]))
    print(case, {k: f"{v:.2e}" for k, v in errs.items()})
    assert errs.pop("u") < FWD_TOL_F32 + spread_u
    for gname, e in errs.items():
        assert e < GRAD_TOL_F32 + spread_g[gname], gname


def _layer(cfg, dtype):
    from ttc_b200 import TTCLayer
    layer = TTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    return layer.to("cuda", dtype)


@pytest.mark.parametrize("case,dtype", [("fused_layer_cfg3", torch.float32),
                                        ("fused_layer_cfg5", torch.float32),
                                        ("fused_layer_cfg5_bf16", torch.bfloat16)])
def test_layer_matches_reference_fused_layer(case, dtype):
    z = load(case)
    cfg = CONFIGS[int(z["cfg"])]
    layer = _layer(cfg, dtype)
    x = torch.from_numpy(z["x"]).to("cuda", dtype)[None].requires_grad_(True)
    y = layer(x, T=int(z["T"]))
    (y[0] * torch.from_numpy(z["dy"]).to("cuda", dtype)).sum().backward()
    fwd_tol, grad_tol = (FWD_TOL_F32, GRAD_TOL_F32) if dtype == torch.float32 else (FWD_TOL_BF16, GRAD_TOL_BF16)
    errs = {"y": O.max_rel(y[0].detach().float().cpu(), torch.from_numpy(z["y"])),
            "x": O.max_rel(x.grad[0].float().cpu(), torch.from_numpy(z["g_x"]))}
    for pn, p in layer.named_parameters():
        s = int(z["stride_" + pn])
        errs[pn] = O.max_rel(p.grad[::s].float().cpu(), torch.from_numpy(z["g_" + pn]))
    print(case, {k: f"{v:.2e}" for k, v in errs.items()})
    assert errs.pop("y") < fwd_tol
    for k, v in errs.items():
        assert v < grad_tol, (k, v)
