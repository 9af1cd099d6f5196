"""Parameter-gradient reductions of the layer's linear maps as batched GEMMs.

The weight gradients of in_proj, out_proj and the low-rank B / Q bases
(ttc_layer.py:53-57,115-123) contract over all N rows of the batch: an (m x K) @ (K x n)
GEMM with K = N (65 536 at config 2) and a small m x n.  In fp32 (no TF32, as the reference
runs) cuBLAS serves such a shape with one split-K kernel; splitting K into C chunks
explicitly and running them as one batched GEMM, then summing the C partial products, is
1.3-3.8x faster on B200 for these shapes (the sum over the chunks is a fixed-order
reduction).  The forward products and the input gradients are plain cuBLAS calls.
"""
from __future__ import annotations

import torch


def _chunks(K: int) -> int:
    """Number of K chunks: up to 64, each at least 256 rows, dividing K; 1 = no split."""
    c = 64
    while c > 1 and (K % c or K // c < 256):
        c //= 2
    return c


def _at_b(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a^T @ b for a [K, m], b [K, n], as a K-chunked batched GEMM."""
    K = a.shape[0]
    c = _chunks(K)
    if c == 1:
        return a.t() @ b
    return torch.bmm(a.reshape(c, K // c, a.shape[1]).transpose(1, 2),
                     b.reshape(c, K // c, b.shape[1])).sum(0)


class _Linear(torch.autograd.Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        y = x @ weight.t()
        return y + bias if bias is not None else y

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, gy):
        x, weight = ctx.saved_tensors
        gx = gy @ weight if ctx.needs_input_grad[0] else None
        gw = _at_b(gy, x) if ctx.needs_input_grad[1] else None
        gb = gy.sum(0) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return gx, gw, gb


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """F.linear for 2-D x [K, in] with the K-chunked weight gradient."""
    return _Linear.apply(x, weight, bias)


class _LowRankMix(torch.autograd.Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, coeff, basis):
        ctx.save_for_backward(coeff, basis)
        r = basis.shape[0]
        return (coeff.reshape(-1, r) @ basis.reshape(r, -1)).view(*coeff.shape[:-1], *basis.shape[1:])

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, g):
        coeff, basis = ctx.saved_tensors
        r = basis.shape[0]
        g2 = g.reshape(-1, basis[0].numel())
        gc = (g2 @ basis.reshape(r, -1).t()).view(coeff.shape) if ctx.needs_input_grad[0] else None
        gb = _at_b(coeff.reshape(-1, r), g2).view(basis.shape) if ctx.needs_input_grad[1] else None
        return gc, gb


def lowrank_mix(coeff: torch.Tensor, basis: torch.Tensor) -> torch.Tensor:
    """einsum("...r,rmn->...mn", coeff, basis) with the K-chunked basis gradient."""
    return _LowRankMix.apply(coeff, basis)
