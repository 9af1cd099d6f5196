"""``solver_impl="cuda"``: the B200 LQR solve behind TTCLayer's solver plug-in point.

The reference picks its solver from a string -> callable map
(ttc/layers/ttc_layer.py:18-22) and calls it as
``solver(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T) -> u``
(ttc_layer.py:137).  ``cuda_lqr_solve`` honours that signature and the behaviour of the
reference's default ``fused`` solver (ttc/solvers/fused_lqr.py:255-304): same shapes and
assertions, fp32 solver state, ``u`` and gradients in the inputs' dtype, symmetrised
Q / Q_f gradients, and the same ``RuntimeError`` messages on NaN, Inf or |x| >= 1e6.

The work runs in two kernels of libttc_b200.so (include/ttc_b200.h): ``ttc_lqr_fwd``
(sweep + LU solve + first step, replacing fused_lqr.py:18-146) and ``ttc_lqr_bwd``
(adjoint, replacing fused_lqr.py:148-253).  There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import torch

from . import _lib

FWD_UNSTABLE_MSG = "Numerical instability detected during fused LQR forward recurrence."
LU_UNSTABLE_MSG = "Numerical instability detected during fused LQR LU solve."
BWD_UNSTABLE_MSG = "Numerical instability detected during fused LQR backward pass."
U_NAN_MSG = "NaN detected in TTC layer solver output."
MMA_TIMEOUT_MSG = ("ttc_b200: a tensor-core MMA did not complete within the kernel's poll limit "
                   "(the launch's results are not valid)")

# The backward needs d_p = Y1^-1 (Y3 du).  The forward keeps M = Y1^-1 Y3
# ([N,nh,d,du] fp32) when it fits this budget, else the backward recomputes the sweep.
SAVE_BUDGET_BYTES = 8 << 30

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


class KernelTimer:
    """Opt-in CUDA-event timing of each solver launch, recorded on the launch stream.
    ``durations_ms()`` synchronises and returns {kernel name: [ms per launch]}."""

    def __init__(self):
        self.pairs: dict[str, list] = {}

    def start(self, stream):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    def stop(self, name, stream, start_ev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        self.pairs.setdefault(name, []).append((start_ev, ev))

    def durations_ms(self):
        torch.cuda.synchronize()
        return {k: [a.elapsed_time(b) for a, b in v] for k, v in self.pairs.items()}


_timer: KernelTimer | None = None


def set_kernel_timer(timer: KernelTimer | None) -> None:
    """Install (or remove with None) the timer the solver launches report to."""
    global _timer
    _timer = timer


def _launch(name, dev, fn, *args):
    stream = torch.cuda.current_stream(dev)
    t = _timer
    ev = t.start(stream) if t is not None else None
    rc = fn(*args, stream.cuda_stream)
    if t is not None:
        t.stop(name, stream, ev)
    _lib.check(rc)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_shapes(A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T):
    """Shape contract of fused_lqr_layer_fwd (ttc/solvers/fused_lqr.py:31-47)."""
    assert T > 0, "T must be positive"
    bs, nh, d = A_diag.shape
    du = B.shape[-1]
    assert B.shape == (bs, d, du), f"B must be [{bs},{d},{du}], got {tuple(B.shape)}"
    assert Q.shape == (bs, d, d), f"Q must be [{bs},{d},{d}], got {tuple(Q.shape)}"
    assert R_inv.shape == (bs, nh, du), f"R_inv must be [{bs},{nh},{du}]"
    assert Q_f.shape == (bs, nh, d, d), f"Q_f must be [{bs},{nh},{d},{d}]"
    assert lgA.shape == (bs, nh), f"log_gamma_A must be [{bs},{nh}]"
    assert lgB.shape == (bs, nh, du), f"log_gamma_B must be [{bs},{nh},{du}]"
    assert lgQ.shape == (bs, nh, d), f"log_gamma_Q must be [{bs},{nh},{d}]"
    assert h0.shape == (bs, nh, d), f"h0 must be [{bs},{nh},{d}]"
    return bs, nh, d, du


def check_fwd_status(st: int) -> None:
    """Raise the reference's forward RuntimeError for the TTC_STATUS_* bits of a forward."""
    if st & _lib.STATUS_MMA_TIMEOUT:
        raise RuntimeError(MMA_TIMEOUT_MSG)
    if st & _lib.STATUS_FWD_UNSTABLE:
        raise RuntimeError(FWD_UNSTABLE_MSG)
    if st & _lib.STATUS_LU_UNSTABLE:
        raise RuntimeError(LU_UNSTABLE_MSG)


def check_bwd_status(st: int) -> None:
    """Raise for the TTC_STATUS_* bits of a backward."""
    if st & _lib.STATUS_MMA_TIMEOUT:
        raise RuntimeError(MMA_TIMEOUT_MSG)
    if st & _lib.STATUS_BWD_UNSTABLE:
        raise RuntimeError(BWD_UNSTABLE_MSG)


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """t itself, or a copy when its data does not start on a 16-byte boundary (the kernels
    read M, d_u and the bases with 16-byte loads)."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _prepare(tensors, dtype):
    out = []
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("ttc_b200 'cuda' solver needs CUDA tensors (there is no CPU path)")
        out.append(_aligned(t.detach().to(dtype).contiguous()))
    return out


class LQRSolveFunction(torch.autograd.Function):
    """Autograd wrapper of ttc_lqr_fwd / ttc_lqr_bwd (mirrors FusedLQRSolveFunc,
    ttc/solvers/fused_lqr.py:255-291).  Returns (u, status) where status is a CPU int32
    tensor carrying the forward's TTC_STATUS_* bits."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T, save_budget, flags=0):
        T = int(T)
        flags = int(flags)
        N, nh, d, du = _check_shapes(A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0, T)
        dtype = Q.dtype
        if dtype not in _DTYPES:
            raise TypeError(f"ttc_b200 'cuda' solver supports float32 and bfloat16, got {dtype}")
        args = _prepare((A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0), dtype)
        dev = Q.device
        lib = _lib.load()
        u = torch.empty(N, nh, du, device=dev, dtype=dtype)
        lam0 = torch.empty(N, nh, d, device=dev, dtype=torch.float32)
        keep_m = N * nh * d * du * 4 <= save_budget
        M = torch.empty(N, nh, d, du, device=dev, dtype=torch.float32) if keep_m else None
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev), torch.profiler.record_function("fwd:ttc_lqr_fwd"):
            _launch("ttc_lqr_fwd", dev, lib.ttc_lqr_fwd, *[_ptr(a) for a in args], N, nh, d, du,
                    T, _DTYPES[dtype], flags, _ptr(u), _ptr(lam0), _ptr(M), _ptr(status))
        st = int(status.item())
        check_fwd_status(st)
        A_c, B_c, Q_c, R_c, Qf_c, lA_c, lB_c, lQ_c, h0_c = args
        ctx.save_for_backward(A_c, B_c, Q_c, R_c, None if keep_m else Qf_c, lA_c, lB_c, lQ_c,
                              h0_c, lam0 if keep_m else None, M)
        ctx.dims = (N, nh, d, du, T)
        ctx.flags = flags
        ctx.dtype = dtype
        ctx.in_dtypes = [t.dtype for t in (A_diag, B, Q, R_inv, Q_f, lgA, lgB, lgQ, h0)]
        status_cpu = torch.tensor([st], dtype=torch.int32)
        ctx.mark_non_differentiable(status_cpu)
        return u, status_cpu

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, d_u, _d_status):
        A, B, Q, R, Qf, lA, lB, lQ, h0, lam0, M = ctx.saved_tensors
        N, nh, d, du, T = ctx.dims
        dtype = ctx.dtype
        dev = Q.device
        d_u = _aligned(d_u.to(dtype).contiguous())
        grads = [torch.empty_like(t) for t in (A, B, Q, R)]
        grads.append(torch.empty(N, nh, d, d, device=dev, dtype=dtype))
        grads += [torch.empty_like(t) for t in (lA, lB, lQ, h0)]
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        lib = _lib.load()
        with torch.cuda.device(dev), torch.profiler.record_function("bwd:ttc_lqr_bwd"):
            _launch("ttc_lqr_bwd", dev, lib.ttc_lqr_bwd,
                    *[_ptr(t) for t in (A, B, Q, R, Qf, lA, lB, lQ, h0)], _ptr(lam0), _ptr(M),
                    _ptr(d_u), N, nh, d, du, T, _DTYPES[dtype], ctx.flags, *[_ptr(g) for g in grads],
                    _ptr(status))
        check_bwd_status(int(status.item()))
        grads = [g.to(dt) for g, dt in zip(grads, ctx.in_dtypes)]
        return (*grads, None, None, None)


def mix_available(N: int, nh: int, d: int, du: int, rQ: int, dtype, save_budget: int | None = None) -> bool:
    """Whether the solve can take Q_f as the layer's rank-r mixture (ttc_lqr_fwd_mix /
    ttc_lqr_bwd_mix): needs the saved-state warp-MMA backward, i.e. M within the budget and a
    supported shape.  Queries the current CUDA device."""
    budget = SAVE_BUDGET_BYTES if save_budget is None else int(save_budget)
    if dtype not in _DTYPES or N == 0 or N * nh * d * du * 4 > budget:
        return False
    return _lib.load().ttc_lqr_bwd_mix_slices(N, nh, d, du, rQ, _DTYPES[dtype]) > 0


class LQRSolveMixFunction(torch.autograd.Function):
    """LQRSolveFunction with Q_f = sum_r coeff_Qf[..., r] Q_basis[r] never materialised
    (ttc_layer.py:119-123 fused into the solve): the forward mixes each head's Q_f rows in the
    kernel, the backward returns grad_coeff_Qf and grad_Q_basis instead of grad_Q_f.  Always
    saves M (callers check ``mix_available`` first)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, A_diag, B, Q, R_inv, coeff_Qf, Q_basis, lgA, lgB, lgQ, h0, T):
        T = int(T)
        N, nh, d = A_diag.shape
        du = B.shape[-1]
        rQ = Q_basis.shape[0]
        assert coeff_Qf.shape == (N, nh, rQ), f"coeff_Qf must be [{N},{nh},{rQ}]"
        assert Q_basis.shape == (rQ, d, d), f"Q_basis must be [{rQ},{d},{d}]"
        dtype = Q.dtype
        if dtype not in _DTYPES:
            raise TypeError(f"ttc_b200 'cuda' solver supports float32 and bfloat16, got {dtype}")
        args = _prepare((A_diag, B, Q, R_inv, coeff_Qf, Q_basis, lgA, lgB, lgQ, h0), dtype)
        dev = Q.device
        lib = _lib.load()
        u = torch.empty(N, nh, du, device=dev, dtype=dtype)
        lam0 = torch.empty(N, nh, d, device=dev, dtype=torch.float32)
        M = torch.empty(N, nh, d, du, device=dev, dtype=torch.float32)
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        A_c, B_c, Q_c, R_c, cQf_c, Qb_c, lA_c, lB_c, lQ_c, h0_c = args
        with torch.cuda.device(dev), torch.profiler.record_function("fwd:ttc_lqr_fwd_mix"):
            _launch("ttc_lqr_fwd", dev, lib.ttc_lqr_fwd_mix, _ptr(A_c), _ptr(B_c), _ptr(Q_c), _ptr(R_c),
                    _ptr(cQf_c), _ptr(Qb_c), rQ, _ptr(lA_c), _ptr(lB_c), _ptr(lQ_c), _ptr(h0_c), N, nh, d,
                    du, T, _DTYPES[dtype], 0, _ptr(u), _ptr(lam0), _ptr(M), _ptr(status))
        st = int(status.item())
        check_fwd_status(st)
        ctx.save_for_backward(*args, lam0, M)
        ctx.dims = (N, nh, d, du, rQ, T)
        ctx.dtype = dtype
        ctx.in_dtypes = [t.dtype for t in (A_diag, B, Q, R_inv, coeff_Qf, Q_basis, lgA, lgB, lgQ, h0)]
        status_cpu = torch.tensor([st], dtype=torch.int32)
        ctx.mark_non_differentiable(status_cpu)
        return u, status_cpu

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, d_u, _d_status):
        A, B, Q, R, cQf, Qb, lA, lB, lQ, h0, lam0, M = ctx.saved_tensors
        N, nh, d, du, rQ, T = ctx.dims
        dtype = ctx.dtype
        dev = Q.device
        lib = _lib.load()
        d_u = _aligned(d_u.to(dtype).contiguous())
        with torch.cuda.device(dev):
            slices = int(lib.ttc_lqr_bwd_mix_slices(N, nh, d, du, rQ, _DTYPES[dtype]))
        if slices <= 0:
            _lib.check(-slices if slices < 0 else _lib.ERR_UNSUPPORTED)
        gA, gB, gQ, gR = [torch.empty_like(t) for t in (A, B, Q, R)]
        gcQf = torch.empty_like(cQf)
        partial = torch.empty(slices, rQ, d, d, device=dev, dtype=torch.float32)
        glA, glB, glQ, gh0 = [torch.empty_like(t) for t in (lA, lB, lQ, h0)]
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev), torch.profiler.record_function("bwd:ttc_lqr_bwd_mix"):
            _launch("ttc_lqr_bwd", dev, lib.ttc_lqr_bwd_mix,
                    *[_ptr(t) for t in (A, B, Q, R, cQf, Qb)], rQ,
                    *[_ptr(t) for t in (lA, lB, lQ, h0)], _ptr(lam0), _ptr(M), _ptr(d_u), N, nh, d, du,
                    T, _DTYPES[dtype], _ptr(gA), _ptr(gB), _ptr(gQ), _ptr(gR), _ptr(gcQf), _ptr(partial),
                    slices, _ptr(glA), _ptr(glB), _ptr(glQ), _ptr(gh0), _ptr(status))
        check_bwd_status(int(status.item()))
        S = partial.sum(0)
        gQb = 0.5 * (S + S.transpose(-1, -2))
        grads = [gA, gB, gQ, gR, gcQf, gQb, glA, glB, glQ, gh0]
        grads = [g.to(dt) for g, dt in zip(grads, ctx.in_dtypes)]
        return (*grads, None)


def lqr_solve_mix_with_status(A_diag, B, Q, R_inv_diag, coeff_Qf, Q_basis, log_gamma_A, log_gamma_B,
                              log_gamma_Q, h0, T):
    """The solve with Q_f given as a mixture (see LQRSolveMixFunction); returns (u, status)."""
    u, status = LQRSolveMixFunction.apply(A_diag, B, Q, R_inv_diag, coeff_Qf, Q_basis, log_gamma_A,
                                          log_gamma_B, log_gamma_Q, h0, T)
    return u, int(status.item())


class LQRSolveLowRankFunction(torch.autograd.Function):
    """The layer's whole low-rank solve (ttc_layer.py:115-137 fused): B = sum_r coeff_B[r]
    B_basis[r], Q = sum_r coeff_Q[r] Q_basis[r] and Q_f = sum_r coeff_Qf[..., r] Q_basis[r]
    are formed inside the kernels (ttc_lqr_fwd_lowrank / ttc_lqr_bwd_lowrank), so none of the
    [N, d, du], [N, d, d] or [N, nh, d, d] tensors exists; the backward returns the gradients of
    the coefficients and the bases.  Saves M when an input needs a gradient (callers check
    ``mix_available`` first)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, A_diag, coeff_B, B_basis, coeff_Q, Q_basis, R_inv, coeff_Qf, lgA, lgB, lgQ, h0, T):
        T = int(T)
        N, nh, d = A_diag.shape
        rB, _, du = B_basis.shape
        rQ = Q_basis.shape[0]
        assert coeff_B.shape == (N, rB), f"coeff_B must be [{N},{rB}]"
        assert coeff_Q.shape == (N, rQ), f"coeff_Q must be [{N},{rQ}]"
        assert coeff_Qf.shape == (N, nh, rQ), f"coeff_Qf must be [{N},{nh},{rQ}]"
        assert Q_basis.shape == (rQ, d, d), f"Q_basis must be [{rQ},{d},{d}]"
        assert B_basis.shape == (rB, d, du), f"B_basis must be [{rB},{d},{du}]"
        dtype = A_diag.dtype
        if dtype not in _DTYPES:
            raise TypeError(f"ttc_b200 'cuda' solver supports float32 and bfloat16, got {dtype}")
        inputs = (A_diag, coeff_B, B_basis, coeff_Q, Q_basis, R_inv, coeff_Qf, lgA, lgB, lgQ, h0)
        args = _prepare(inputs, dtype)
        A_c, cB_c, Bb_c, cQ_c, Qb_c, R_c, cQf_c, lA_c, lB_c, lQ_c, h0_c = args
        dev = A_diag.device
        lib = _lib.load()
        keep = any(ctx.needs_input_grad[:11])
        u = torch.empty(N, nh, du, device=dev, dtype=dtype)
        lam0 = torch.empty(N, nh, d, device=dev, dtype=torch.float32) if keep else None
        M = torch.empty(N, nh, d, du, device=dev, dtype=torch.float32) if keep else None
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev), torch.profiler.record_function("fwd:ttc_lqr_fwd_lowrank"):
            _launch("ttc_lqr_fwd", dev, lib.ttc_lqr_fwd_lowrank, _ptr(A_c), _ptr(cB_c), _ptr(Bb_c), rB,
                    _ptr(cQ_c), _ptr(R_c), _ptr(cQf_c), _ptr(Qb_c), rQ, _ptr(lA_c), _ptr(lB_c), _ptr(lQ_c),
                    _ptr(h0_c), N, nh, d, du, T, _DTYPES[dtype], 0, _ptr(u), _ptr(lam0), _ptr(M), _ptr(status))
        st = int(status.item())
        check_fwd_status(st)
        if keep:
            ctx.save_for_backward(*args, lam0, M)
        ctx.dims = (N, nh, d, du, rB, rQ, T)
        ctx.dtype = dtype
        ctx.in_dtypes = [t.dtype for t in inputs]
        status_cpu = torch.tensor([st], dtype=torch.int32)
        ctx.mark_non_differentiable(status_cpu)
        return u, status_cpu

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, d_u, _d_status):
        A, cB, Bb, cQ, Qb, R, cQf, lA, lB, lQ, h0, lam0, M = ctx.saved_tensors
        N, nh, d, du, rB, rQ, T = ctx.dims
        dtype = ctx.dtype
        dev = A.device
        lib = _lib.load()
        d_u = _aligned(d_u.to(dtype).contiguous())
        with torch.cuda.device(dev):
            slices = int(lib.ttc_lqr_bwd_mix_slices(N, nh, d, du, rQ, _DTYPES[dtype]))
        if slices <= 0:
            _lib.check(-slices if slices < 0 else _lib.ERR_UNSUPPORTED)
        gA, gcB, gcQ, gR, gcQf, glA, glB, glQ, gh0 = [torch.empty_like(t) for t in (A, cB, cQ, R, cQf, lA, lB, lQ, h0)]
        part_q = torch.empty(slices, rQ, d, d, device=dev, dtype=torch.float32)
        part_b = torch.empty(slices, rB, d, du, device=dev, dtype=torch.float32)
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        with torch.cuda.device(dev), torch.profiler.record_function("bwd:ttc_lqr_bwd_lowrank"):
            _launch("ttc_lqr_bwd", dev, lib.ttc_lqr_bwd_lowrank, _ptr(A), _ptr(cB), _ptr(Bb), rB, _ptr(cQ),
                    _ptr(R), _ptr(cQf), _ptr(Qb), rQ, _ptr(lA), _ptr(lB), _ptr(lQ), _ptr(h0), _ptr(lam0),
                    _ptr(M), _ptr(d_u), N, nh, d, du, T, _DTYPES[dtype], _ptr(gA), _ptr(gcB), _ptr(part_b),
                    _ptr(gcQ), _ptr(gR), _ptr(gcQf), _ptr(part_q), slices, _ptr(glA), _ptr(glB), _ptr(glQ),
                    _ptr(gh0), _ptr(status))
        check_bwd_status(int(status.item()))
        S = part_q.sum(0)
        gQb = 0.5 * (S + S.transpose(-1, -2))
        gBb = part_b.sum(0)
        grads = [gA, gcB, gBb, gcQ, gQb, gR, gcQf, glA, glB, glQ, gh0]
        grads = [g.to(dt) for g, dt in zip(grads, ctx.in_dtypes)]
        return (*grads, None)


def lqr_solve_lowrank_with_status(A_diag, coeff_B, B_basis, coeff_Q, Q_basis, R_inv_diag, coeff_Qf,
                                  log_gamma_A, log_gamma_B, log_gamma_Q, h0, T):
    """The solve with B, Q and Q_f given as the layer's mixtures (see LQRSolveLowRankFunction);
    returns (u, status)."""
    u, status = LQRSolveLowRankFunction.apply(A_diag, coeff_B, B_basis, coeff_Q, Q_basis, R_inv_diag,
                                              coeff_Qf, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T)
    return u, int(status.item())


def _flags(inv_guard: bool) -> int:
    return _lib.FLAG_INV_GUARD if inv_guard else 0


def lqr_solve_with_status(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q,
                          h0, T, save_budget: int | None = None, inv_guard: bool = False):
    """Like ``cuda_lqr_solve`` but also returns the forward's status bits (host int)."""
    budget = SAVE_BUDGET_BYTES if save_budget is None else int(save_budget)
    u, status = LQRSolveFunction.apply(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B,
                                       log_gamma_Q, h0, T, budget, _flags(inv_guard))
    return u, int(status.item())


def cuda_lqr_solve(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B, log_gamma_Q, h0, T,
                   save_budget: int | None = None, inv_guard: bool = False, num_chunks: int = 1):
    """Drop-in for the reference solvers (ttc_layer.py:137): returns u [N, nh, du].

    ``inv_guard`` adds 1e-6 I to Y1 before the solve, as the reference's fused solver
    (fused_lqr.py:294-304).  ``num_chunks`` is the horizon split of fused_lqr_layer_fwd
    (fused_lqr.py:26-35, T divisible by it); the kernels keep the recurrence state on chip for
    the whole horizon with each step's own discount exponent, so every split gives the
    unchunked result."""
    assert T > 0 and T % num_chunks == 0, "T must be a positive multiple of num_chunks"
    return lqr_solve_with_status(A_diag, B, Q, R_inv_diag, Q_f, log_gamma_A, log_gamma_B,
                                 log_gamma_Q, h0, T, save_budget, inv_guard)[0]


def fused_lqr_solve(A_diag, B, Q, R_inv_diag, Q_f, gamma_A, gamma_B, gamma_Q, h0, T,
                    inv_guard: bool = False):
    """The reference's public fused entry point (fused_lqr.py:294-304), same signature."""
    return cuda_lqr_solve(A_diag, B, Q, R_inv_diag, Q_f, gamma_A, gamma_B, gamma_Q, h0, T,
                          inv_guard=inv_guard)


def kkt_lqr_solve(A_diag, B, Q, R_inv_diag, Q_f, gamma_A, gamma_B, gamma_Q, h0, T,
                  save_budget: int | None = None):
    """The reference's ``kkt`` solver on the GPU (see ttc_b200.kkt)."""
    from .kkt import kkt_lqr_solve as impl
    return impl(A_diag, B, Q, R_inv_diag, Q_f, gamma_A, gamma_B, gamma_Q, h0, T, save_budget)


# The plug-in map of ttc_layer.py:18-22.  "fused" (the reference's default name) maps to
# the CUDA solver so TTCLayer(..., solver_impl="fused") keeps working after the switch;
# "kkt" is the reference's kkt solver (Riccati forward, two-problem backward) on the GPU.
# The reference's "riccati" (autograd through the Riccati recursion, whose Q gradient is not
# symmetrised) is the CPU oracle and has no GPU entry.
LQR_SOLVER_IMPL_MAP = {
    "cuda": cuda_lqr_solve,
    "fused": cuda_lqr_solve,
    "kkt": kkt_lqr_solve,
}
