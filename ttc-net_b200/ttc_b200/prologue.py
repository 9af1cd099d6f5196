"""The layer's elementwise prologue on the GPU: one CUDA kernel forward, one backward.

Between in_proj and the low-rank einsums, TTCLayer.forward (ttc/layers/ttc_layer.py:106-133)
splits the projection Z into per-head and per-row pieces and applies l2norm / softplus /
clamp / negation to them.  As separate PyTorch ops that is ~20 launches forward and ~30
backward (plus the concatenation of the split's gradient), all reading and writing Z-sized
tensors.  ``prologue`` does the same arithmetic in ``ttc_prologue_fwd`` (rows of Z staged in
shared memory by bulk copies when they are 16-byte aligned) and its chain rule in
``ttc_prologue_bwd`` (include/ttc_b200.h), with the reference's roundings in bf16.  No
fallback: without the CUDA library these raise.
"""
from __future__ import annotations

import torch

from . import _lib
from .solver import _DTYPES, _launch, _ptr


class PrologueFunction(torch.autograd.Function):
    """Z [N, W] -> (A_diag, R_inv, coeff_Qf, lgA, lgB, lgQ, h0, coeff_B, coeff_Q)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, Z, nh, d, du, rB, rQ):
        if Z.dtype not in _DTYPES:
            raise TypeError(f"ttc_b200 prologue: unsupported dtype {Z.dtype}")
        if not Z.is_cuda:
            raise RuntimeError("ttc_b200 prologue needs a CUDA tensor")
        Z = Z.contiguous()
        N = Z.shape[0]
        assert Z.shape[1] == nh * (4 * d + 2 * du + 1) + rB + rQ, "in_proj width mismatch"
        kw = dict(device=Z.device, dtype=Z.dtype)
        outs = (torch.empty(N, nh, d, **kw), torch.empty(N, nh, du, **kw), torch.empty(N, nh, d, **kw),
                torch.empty(N, nh, **kw), torch.empty(N, nh, du, **kw), torch.empty(N, nh, d, **kw),
                torch.empty(N, nh, d, **kw), torch.empty(N, rB, **kw), torch.empty(N, rQ, **kw))
        lib = _lib.load()
        status = torch.zeros(1, device=Z.device, dtype=torch.int32)
        _launch("ttc_prologue_fwd", Z.device, lib.ttc_prologue_fwd, _ptr(Z), N, nh, d, du, rB, rQ,
                _DTYPES[Z.dtype], *[_ptr(o) for o in outs], _ptr(status))
        ctx.save_for_backward(Z)
        ctx.dims = (nh, d, du, rB, rQ)
        _pending.append(status)
        if len(_pending) > 64:  # callers that never check: keep the list bounded
            check_status()
        return outs

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, *grads):
        (Z,) = ctx.saved_tensors
        nh, d, du, rB, rQ = ctx.dims
        gs = [None if g is None else g.to(Z.dtype).contiguous() for g in grads]
        dZ = torch.empty_like(Z)
        lib = _lib.load()
        _launch("ttc_prologue_bwd", Z.device, lib.ttc_prologue_bwd, _ptr(Z), Z.shape[0], nh, d, du, rB,
                rQ, _DTYPES[Z.dtype], *[_ptr(g) for g in gs], _ptr(dZ))
        return dZ, None, None, None, None, None


# Status words of forward launches not checked yet.  The layer reads them after its solver's
# own status read has synchronised the stream, so the check adds a copy but no wait.
_pending: list = []


def check_status() -> None:
    """Raise if a prologue forward since the last check reported a stalled bulk copy."""
    global _pending
    words, _pending = _pending, []
    for w in words:
        if int(w.item()) & _lib.STATUS_COPY_TIMEOUT:
            raise RuntimeError(COPY_TIMEOUT_MSG)


COPY_TIMEOUT_MSG = ("ttc_b200: a bulk copy of the projection into shared memory did not complete within "
                    "the prologue kernel's wait limit (its outputs are not valid)")


def prologue(Z: torch.Tensor, nh: int, d: int, du: int, rB: int, rQ: int):
    return PrologueFunction.apply(Z, nh, d, du, rB, rQ)
