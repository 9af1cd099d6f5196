"""TTCLayer with the B200 LQR solver -- a drop-in for ttc.TTCLayer
(ttc/layers/ttc_layer.py:24-153): same constructor signature, parameter names, shapes
and initialisation, so a reference ``state_dict`` loads 1:1.

The prologue's elementwise part (split, l2norm / softplus / clamp, ttc_layer.py:106-133)
runs as one CUDA kernel each way (``prologue.py``); the low-rank mixtures of B, Q and the
per-head Q_f (:115-123) are formed inside the solver kernels when the saved-state backward
applies (``mix_available``), so no [N, d, du] B, [N, d, d] Q or [N, nh, d, d] Q_f tensor (nor
their gradients) exists; the epilogue's l2norm of u (:142-143) is one CUDA kernel each way
(``epilogue.py``); in_proj and out_proj are cuBLAS GEMMs; the LQR solve runs in
libttc_b200.so through ``LQR_SOLVER_IMPL_MAP``.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .epilogue import rownorm
from .prologue import check_status as check_prologue_status
from .prologue import prologue
from .reductions import linear, lowrank_mix
from .solver import (LQR_SOLVER_IMPL_MAP, U_NAN_MSG, cuda_lqr_solve, lqr_solve_lowrank_with_status,
                     lqr_solve_with_status, mix_available)
from . import _lib


# Device memory one layer call may keep for its backward (in_proj output, prologue outputs,
# B / Q mixtures, the solver's saved state), capped further at half the free memory when the
# call starts.  Larger inputs run in row chunks (see TTCLayer.forward).
CALL_BUDGET_BYTES = 24 << 30


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x / sqrt(sum(x^2) + eps) over the last dim in fp32, cast back (the formula of
    fla.modules.l2norm used by the reference, fla/modules/l2norm.py:42)."""
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


class TTCLayer(nn.Module):
    def __init__(self, in_dim: int, out_dim: int, h_dim: int, num_heads: int,
                 b_rank: int, q_rank: int, u_dim: int | None = None,
                 bias: bool = False, gamma_bias: bool = False, gamma_bias_init: str = "sqrt_dim",
                 rescale: str = "l2_norm", q_reparam: str = "plain", solver_impl: str = "cuda"):
        super().__init__()
        if u_dim is None:
            u_dim = h_dim
        assert solver_impl in LQR_SOLVER_IMPL_MAP, f"Unknown LQR solver {solver_impl}"
        self.solver_impl = solver_impl
        self.solver = LQR_SOLVER_IMPL_MAP[solver_impl]
        assert rescale in ["none", "l2_norm", "h0_norm"], f"Unknown rescale method {rescale}"
        self.rescale = rescale
        self.q_reparam = q_reparam
        assert q_reparam in ["plain", "cholesky"], f"Unknown Q reparameterization {q_reparam}"
        self.in_dim, self.out_dim, self.num_heads = in_dim, out_dim, num_heads
        self.h_dim, self.u_dim, self.q_rank, self.b_rank = h_dim, u_dim, q_rank, b_rank

        # Per-token projection: headwise [h0, A_diag, R_inv_diag, Qf coeffs, log-gammas]
        # and the shared B / Q basis coefficients (ttc_layer.py:53-57).
        self.in_proj = nn.Linear(in_dim, (4 * h_dim + 2 * u_dim + 1) * num_heads + b_rank + q_rank,
                                 bias=bias)
        self.out_proj = nn.Linear(u_dim * num_heads, out_dim, bias=bias)
        self.Bs = nn.Parameter(torch.empty(b_rank, h_dim, u_dim))
        self.Qs = nn.Parameter(torch.empty(q_rank, h_dim, h_dim))
        self.ttc_gamma_bias_init = gamma_bias_init
        assert gamma_bias_init in ["sqrt_dim", "zero"], f"Unknown gamma bias initialization {gamma_bias_init}"
        self.bias_gamma = None
        if gamma_bias:
            self.bias_gamma = nn.Parameter(torch.empty(1 + u_dim + h_dim, dtype=torch.float32))
        TTCLayer._init_module(self)

    @staticmethod
    def _init_module(module, std=0.02):
        """ttc_layer.py:72-96."""
        with torch.no_grad():
            module.Bs.data.normal_(mean=0.0, std=std)
            if module.q_reparam == "plain":
                g = torch.empty_like(module.Qs).normal_(mean=0.0, std=std)
                module.Qs.data.copy_(g @ g.transpose(1, 2) / math.sqrt(module.h_dim))
            else:
                module.Qs.data.normal_(mean=0.0, std=std)
            if module.bias_gamma is not None:
                if module.ttc_gamma_bias_init == "sqrt_dim":
                    module.bias_gamma.data.fill_(math.log(1 / math.sqrt(module.h_dim)))
                else:
                    module.bias_gamma.data.fill_(0.0)

    def lowrank_inputs(self, x2d: torch.Tensor):
        """Prologue (ttc_layer.py:104-135) up to, not including, the low-rank mixtures: rows
        [N, in_dim] -> (A_diag, coeff_B, B_basis, coeff_Q, Q_basis, R_inv, coeff_Qf, lgA, lgB,
        lgQ, h0) with B = sum_r coeff_B[..., r] B_basis[r], Q = sum_r coeff_Q[..., r]
        Q_basis[r] and Q_f = sum_r coeff_Qf[..., r] Q_basis[r].  in_proj is a cuBLAS GEMM with
        a K-chunked weight gradient (``reductions``); the elementwise split / l2norm / softplus
        / clamp / negation is one CUDA kernel each way (``prologue``).  Q_basis is the layer's
        Qs, or Qs Qs^T / sqrt(h_dim) for its cholesky reparametrisation (:121-123)."""
        nh, d, du = self.num_heads, self.h_dim, self.u_dim
        A_diag, R_inv_diag, coeff_Qf, log_gamma_A, log_gamma_B, log_gamma_Q, h0, coeff_B, coeff_Q = \
            prologue(linear(x2d, self.in_proj.weight, self.in_proj.bias), nh, d, du, self.b_rank, self.q_rank)
        if self.q_reparam == "plain":
            Q_basis = self.Qs
        else:
            Q_basis = torch.einsum("rmn,rkn->rmk", self.Qs, self.Qs) / math.sqrt(d)
        if self.bias_gamma is not None:
            # log_gammas = -softplus(.) - relu(-bias_gamma), split as [1, du, d] (:129-133)
            bg = F.relu(-self.bias_gamma)
            log_gamma_A = log_gamma_A - bg[0]
            log_gamma_B = log_gamma_B - bg[1:1 + du]
            log_gamma_Q = log_gamma_Q - bg[1 + du:]
        return (A_diag, coeff_B, self.Bs, coeff_Q, Q_basis, R_inv_diag, coeff_Qf, log_gamma_A, log_gamma_B,
                log_gamma_Q, h0)

    @staticmethod
    def _mix(parts):
        """Low-rank parts -> (A_diag, B, Q, R_inv, coeff_Qf, Q_basis, lgA, lgB, lgQ, h0): B and Q
        mixed by cuBLAS GEMMs (the einsums of ttc_layer.py:115-123)."""
        A_diag, coeff_B, B_basis, coeff_Q, Q_basis, R_inv, coeff_Qf, lgA, lgB, lgQ, h0 = parts
        return (A_diag, lowrank_mix(coeff_B, B_basis), lowrank_mix(coeff_Q, Q_basis), R_inv, coeff_Qf,
                Q_basis, lgA, lgB, lgQ, h0)

    def mixed_inputs(self, x2d: torch.Tensor):
        """(A_diag, B, Q, R_inv, coeff_Qf, Q_basis, lgA, lgB, lgQ, h0): the prologue with B and Q
        formed, Q_f still as its mixture."""
        return self._mix(self.lowrank_inputs(x2d))

    @staticmethod
    def _materialise(parts):
        A_diag, B, Q, R_inv, coeff_Qf, Q_basis, lgA, lgB, lgQ, h0 = parts
        Q_f = lowrank_mix(coeff_Qf, Q_basis)
        return (A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0)

    def solver_inputs(self, x2d: torch.Tensor):
        """The nine inputs of the reference solver signature (ttc_layer.py:137), Q_f
        materialised as [N, nh, d, d]."""
        return self._materialise(self.mixed_inputs(x2d))

    def call_bytes_per_row(self, dtype: torch.dtype) -> int:
        """Upper estimate of the device memory one row of a layer call keeps until its
        backward: in_proj output, prologue outputs, B / Q mixtures, Q_f where it is
        materialised, and the solver's saved state (lambda0 and M in fp32)."""
        es = 2 if dtype == torch.bfloat16 else 4
        nh, d, du = self.num_heads, self.h_dim, self.u_dim
        width = self.in_proj.out_features
        return es * (3 * width + 4 * nh * d * d + 3 * d * du + 3 * d * d) + 4 * nh * (4 * d + d * du)

    def rows_per_call(self, N: int, dtype: torch.dtype, device: torch.device) -> int:
        """Rows one layer call takes so that its saved state stays within CALL_BUDGET_BYTES
        and half the device's free memory."""
        budget = CALL_BUDGET_BYTES
        if device.type == "cuda":
            free, _ = torch.cuda.mem_get_info(device)
            budget = min(budget, free // 2)
        return max(1, min(N, budget // self.call_bytes_per_row(dtype)))

    def forward(self, h0: torch.Tensor, T: int) -> torch.Tensor:
        """y = layer(x, T).  x is [bs, seq, in_dim] as in the reference; a 4-D
        [B, L, H, in_dim] input is read as [B, L*H, in_dim] rows and returned as
        [B, L, H, out_dim].

        Rows are independent.  When the whole input would keep more than
        ``rows_per_call`` rows of backward state, the rows run in chunks of that size, each
        under activation checkpointing: the forward keeps only the chunk's input, and the
        backward recomputes one chunk at a time (prologue and solve) before differentiating
        it, so memory stays bounded at any batch size (config 5, 8.4 M rows, on one GPU)."""
        if h0.dim() == 4:
            b, l, hh, _ = h0.shape
            return self.forward(h0.reshape(b, l * hh, -1), T).reshape(b, l, hh, self.out_dim)
        if T == 0:
            return torch.zeros(h0.shape[0], h0.shape[1], self.out_dim, device=h0.device, dtype=h0.dtype)
        bs, seq_len, in_dim = h0.shape
        x2d = h0.reshape(-1, in_dim)
        N = x2d.shape[0]
        rows = self.rows_per_call(N, x2d.dtype, x2d.device) if x2d.is_cuda else N
        if rows >= N:
            return self._forward_rows(x2d, T).view(bs, seq_len, -1)
        keep = torch.is_grad_enabled() and (x2d.requires_grad or any(p.requires_grad for p in self.parameters()))
        outs = []
        for s in range(0, N, rows):
            xs = x2d[s:s + rows]
            if keep:
                outs.append(checkpoint(self._forward_rows, xs, T, use_reentrant=False))
            else:
                outs.append(self._forward_rows(xs, T))
        return torch.cat(outs).view(bs, seq_len, -1)

    def forward_backward(self, x: torch.Tensor, dy: torch.Tensor, T: int, rows: int | None = None,
                         before_last_backward=None) -> torch.Tensor:
        """Forward and backward of the layer over row micro-batches (gradient accumulation):
        each micro-batch of ``rows`` rows (default ``rows_per_call``) runs forward and is
        immediately differentiated with its slice of the upstream gradient ``dy``, so its
        saved state is freed before the next one starts.  Parameter gradients accumulate into
        ``.grad`` and, when ``x`` requires grad, into ``x.grad``, exactly as one
        ``layer(x, T).backward(dy)`` would; returns y (detached), shaped like ``layer(x, T)``.
        ``before_last_backward`` (optional) is called just before the backward that completes
        the parameter gradients (e.g. ``OverlappedGradAllReduce.arm``)."""
        if T == 0:  # y = 0 whatever the parameters (ttc_layer.py:101-102): no gradient
            return torch.zeros(*x.shape[:-1], self.out_dim, device=x.device, dtype=x.dtype)
        in_dim = x.shape[-1]
        x2d = x.reshape(-1, in_dim)
        dy2d = dy.reshape(-1, self.out_dim)
        N = x2d.shape[0]
        if rows is None:
            rows = self.rows_per_call(N, x2d.dtype, x2d.device)
        y = torch.empty(N, self.out_dim, device=x.device, dtype=x.dtype)
        for s in range(0, N, rows):
            ys = self._forward_rows(x2d[s:s + rows], T)
            if before_last_backward is not None and s + rows >= N:
                before_last_backward()
            ys.backward(dy2d[s:s + rows])
            y[s:s + rows] = ys.detach()
        return y.view(*x.shape[:-1], self.out_dim)

    def _forward_rows(self, x2d: torch.Tensor, T: int) -> torch.Tensor:
        """The layer on rows x2d [N, in_dim] -> y [N, out_dim] (ttc_layer.py:104-153)."""
        parts = self.lowrank_inputs(x2d)
        if self.solver is cuda_lqr_solve:
            N, nh, d = parts[0].shape
            if mix_available(N, nh, d, self.u_dim, parts[4].shape[0], parts[0].dtype):
                # B, Q and Q_f mixed inside the kernels: no [N, d, du], [N, d, d] or
                # [N, nh, d, d] tensor either way.
                u, status = lqr_solve_lowrank_with_status(*parts, T)
            else:
                u, status = lqr_solve_with_status(*self._materialise(self._mix(parts)), T)
            check_prologue_status()  # after the solver's status read: no extra wait
            if status & _lib.STATUS_U_NAN:
                raise RuntimeError(U_NAN_MSG)
        else:
            u = self.solver(*self._materialise(self._mix(parts)), T)
            if torch.isnan(u).any():
                raise RuntimeError(U_NAN_MSG)
            check_prologue_status()
        if self.rescale == "l2_norm":
            u = rownorm(u)
        elif self.rescale == "h0_norm":
            x0 = parts[-1]
            h0_norm = torch.linalg.norm(x0, dim=-1, ord=2).detach()
            u_norm = torch.linalg.norm(u, dim=-1, ord=2).detach()
            u = u / u_norm[..., None] * h0_norm[..., None]
        return linear(u.reshape(u.shape[0], -1), self.out_proj.weight, self.out_proj.bias)
