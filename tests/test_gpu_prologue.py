"""GPU parity of the fused layer prologue (ttc_prologue_fwd / ttc_prologue_bwd) against the
PyTorch ops it replaces (ttc/layers/ttc_layer.py:106-133 as split / l2norm / softplus /
clamp / neg), forward outputs and the backward's dZ, fp32 and bf16."""
import pytest
import torch
from prologue_ref import prologue_torch

pytestmark = pytest.mark.gpu


# rows of 16-byte multiples (bulk-copy path: the config-1, -2, -3 and -4 widths) and others
SHAPES = [(512, 16, 16, 16, 16, 16), (77, 3, 16, 16, 16, 16), (300, 5, 32, 32, 32, 32),
          (64, 3, 64, 64, 64, 64), (100, 2, 16, 32, 8, 24), (40, 3, 32, 16, 64, 32),
          (200, 8, 16, 16, 16, 16), (1000, 32, 32, 32, 32, 32), (37, 32, 64, 64, 64, 64)]


def _z(N, nh, d, du, rB, rQ, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = nh * (4 * d + 2 * du + 1) + rB + rQ
    Z = torch.randn(N, W, device="cuda", generator=g) * 3.0
    Z[:, ::17] = 25.0 * torch.sign(Z[:, ::17])  # beyond the softplus threshold both ways
    return Z.to(dtype)


def _maxrel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype,tol_f,tol_b", [(torch.float32, 2e-6, 2e-5), (torch.bfloat16, 1e-2, 2e-2)])
@pytest.mark.parametrize("shape", SHAPES)
def test_prologue_matches_torch(shape, dtype, tol_f, tol_b):
    from ttc_b200.prologue import prologue
    N, nh, d, du, rB, rQ = shape
    Z = _z(*shape, dtype, seed=N + nh)
    Zr = Z.clone().requires_grad_(True)
    Zc = Z.clone().requires_grad_(True)
    ref = prologue_torch(Zr, nh, d, du, rB, rQ)
    out = prologue(Zc, nh, d, du, rB, rQ)
    names = ["A_diag", "R_inv", "coeff_Qf", "lgA", "lgB", "lgQ", "h0", "coeff_B", "coeff_Q"]
    for n, a, b in zip(names, out, ref):
        assert a.shape == b.shape and a.dtype == b.dtype, n
        assert _maxrel(a, b) <= tol_f, f"{n}: {_maxrel(a, b):.2e}"
    g = torch.Generator(device="cuda").manual_seed(7)
    grads = [torch.randn(t.shape, device="cuda", generator=g).to(dtype) for t in ref]
    grads[3] = None  # an output without gradient (e.g. unused) reads as zero
    torch.autograd.backward([t for t, gg in zip(ref, grads) if gg is not None],
                            [gg for gg in grads if gg is not None])
    torch.autograd.backward([t for t, gg in zip(out, grads) if gg is not None],
                            [gg for gg in grads if gg is not None])
    assert _maxrel(Zc.grad, Zr.grad) <= tol_b, f"dZ: {_maxrel(Zc.grad, Zr.grad):.2e}"


def test_prologue_deterministic_and_empty():
    from ttc_b200.prologue import prologue
    N, nh, d, du, rB, rQ = 256, 16, 16, 16, 16, 16
    Z = _z(N, nh, d, du, rB, rQ, torch.float32, seed=3).requires_grad_(True)
    outs = prologue(Z, nh, d, du, rB, rQ)
    sum(o.sum() for o in outs).backward()
    g1 = Z.grad.clone()
    Z.grad = None
    outs2 = prologue(Z, nh, d, du, rB, rQ)
    sum(o.sum() for o in outs2).backward()
    assert torch.equal(g1, Z.grad)
    for a, b in zip(outs, outs2):
        assert torch.equal(a, b)
    empty = prologue(torch.empty(0, Z.shape[1], device="cuda"), nh, d, du, rB, rQ)
    assert empty[0].shape == (0, nh, d)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("shape", [(1000, 32, 32, 32, 32, 32), (3001, 16, 16, 16, 16, 16), (5, 8, 16, 16, 16, 16)])
def test_prologue_bulk_copy_path_equals_direct_loads(shape, dtype):
    """The forward with its rows staged in shared memory by bulk copies (status word given,
    aligned rows) writes bitwise the outputs of the direct-load kernel (no status word)."""
    from ttc_b200 import _lib
    from ttc_b200.solver import _DTYPES
    lib = _lib.load()
    N, nh, d, du, rB, rQ = shape
    Z = _z(*shape, dtype, seed=N)
    assert (Z.shape[1] * Z.element_size()) % 16 == 0 and Z.data_ptr() % 16 == 0

    def run(with_status):
        kw = dict(device="cuda", dtype=dtype)
        outs = [torch.full(s_, float("nan"), **kw) for s_ in
                ((N, nh, d), (N, nh, du), (N, nh, d), (N, nh), (N, nh, du), (N, nh, d), (N, nh, d), (N, rB), (N, rQ))]
        status = torch.zeros(1, device="cuda", dtype=torch.int32) if with_status else None
        rc = lib.ttc_prologue_fwd(Z.data_ptr(), N, nh, d, du, rB, rQ, _DTYPES[dtype], *[o.data_ptr() for o in outs],
                                  None if status is None else status.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.ttc_last_error()
        torch.cuda.synchronize()
        if status is not None:
            assert int(status.item()) == 0
        return outs

    for a, b in zip(run(True), run(False)):
        assert torch.equal(a, b)
