"""The layer prologue as plain PyTorch ops (ttc/layers/ttc_layer.py:106-133 without
bias_gamma): the comparison target of the fused CUDA prologue, and the stand-in for it
when the CPU tests run the product layer's host code without a GPU."""
import torch
import torch.nn.functional as F


def _l2norm(x, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


def prologue_torch(Z, nh, d, du, rB, rQ):
    """The reference's prologue as PyTorch ops (ttc_layer.py:106-133, without bias_gamma)."""
    head_split = [d, d, du, d, 1 + du + d]
    heads, cB, cQ = torch.split(Z, [sum(head_split) * nh, rB, rQ], dim=-1)
    h0, A, R, cQf, lg = torch.split(heads.reshape(-1, nh, sum(head_split)), head_split, dim=-1)
    A = _l2norm(A)
    cB, cQ, cQf = _l2norm(cB), _l2norm(F.softplus(cQ)), _l2norm(F.softplus(cQf))
    R = torch.clamp(_l2norm(F.softplus(R)), min=1e-6)
    lg = -F.softplus(lg)
    lgA, lgB, lgQ = torch.split(lg, [1, du, d], dim=-1)
    return A, R, cQf, lgA.squeeze(-1), lgB, lgQ, h0, cB, cQ
