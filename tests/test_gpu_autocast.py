"""TTCLayer under torch.autocast(bf16) on the GPU: the reference's fused solver runs its
forward and backward with the ambient autocast state (fused_lqr.py:259,281, torch.amp
custom_fwd / custom_bwd), and nn.Linear / einsum autocast to bf16, so a reference user can
train the layer in autocast.  Here the custom autograd Functions carry the same decorators;
the layer must run forward and backward under autocast and agree with the reference's fp32
outputs at the bf16 bar (2e-2 on y), with gradients within 5e-2."""
import numpy as np
import pytest
import torch

from oracle import ttc_oracle as O
from ttc_cases import CONFIGS, layer_weights

pytestmark = pytest.mark.gpu


def _golden(name):
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", name + ".npz"))
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("case", ["layer_cfg2"])
def test_layer_trains_under_autocast(case):
    from ttc_b200 import TTCLayer
    z = _golden(case)
    cfg = CONFIGS[int(z["cfg"])]
    layer = TTCLayer(cfg.in_dim, cfg.out_dim, cfg.h_dim, cfg.H, cfg.rank, cfg.rank)
    layer.load_state_dict({k: torch.from_numpy(v) for k, v in layer_weights(cfg).items()})
    layer = layer.cuda()
    x = torch.from_numpy(z["x"]).cuda()[None].requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = layer(x, T=int(z["T"]))
    assert y.dtype == torch.bfloat16
    assert O.max_rel(y[0].detach().float().cpu(), torch.from_numpy(z["y"])) < 2e-2
    (y[0].float() * torch.from_numpy(z["dy"]).cuda()).sum().backward()
    assert x.grad.dtype == torch.float32
    assert O.max_rel(x.grad[0].cpu(), torch.from_numpy(z["g_x"])) < 5e-2
    for pn, p in layer.named_parameters():
        assert p.grad.dtype == torch.float32, pn
        s = int(z["stride_" + pn])
        assert O.max_rel(p.grad[::s].cpu(), torch.from_numpy(z["g_" + pn])) < 5e-2, pn
