"""The layer's epilogue normalisation on the GPU: l2norm of each head's action vector u
(ttc/layers/ttc_layer.py:142-143, the fla l2norm x rsqrt(sum x^2 + 1e-6) computed in fp32,
fla/modules/l2norm.py:42), one CUDA kernel forward (``ttc_rownorm_fwd``) and one backward
(``ttc_rownorm_bwd``, which recomputes the norm from x instead of saving it).  No fallback:
without the CUDA library these raise.
"""
from __future__ import annotations

import torch

from . import _lib
from .solver import _DTYPES, _launch, _ptr


class RowNormFunction(torch.autograd.Function):
    """x [..., n] -> x / sqrt(sum x^2 + 1e-6) over the last dim (n <= 64)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, x):
        if x.dtype not in _DTYPES:
            raise TypeError(f"ttc_b200 rownorm: unsupported dtype {x.dtype}")
        if not x.is_cuda:
            raise RuntimeError("ttc_b200 rownorm needs a CUDA tensor")
        x = x.contiguous()
        y = torch.empty_like(x)
        n = x.shape[-1]
        rows = x.numel() // n if n else 0
        _launch("ttc_rownorm_fwd", x.device, _lib.load().ttc_rownorm_fwd, _ptr(x), rows, n,
                _DTYPES[x.dtype], _ptr(y))
        ctx.save_for_backward(x)
        return y

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        g = g.to(x.dtype).contiguous()
        dx = torch.empty_like(x)
        n = x.shape[-1]
        rows = x.numel() // n if n else 0
        _launch("ttc_rownorm_bwd", x.device, _lib.load().ttc_rownorm_bwd, _ptr(x), _ptr(g), rows, n,
                _DTYPES[x.dtype], _ptr(dx))
        return dx


def rownorm(x: torch.Tensor) -> torch.Tensor:
    return RowNormFunction.apply(x)
