"""ttc_lqr_bwd_mix_noalloc, the allocation-free variant of the mixed-Q_f backward, against the
allocating entry point it stands in for (ttc_lqr_bwd_mix + the caller's slice sum), through
the C-ABI.

The variant exists for callers that cannot allocate device memory (a host runtime that owns
all device memory in its own pool, or a latency-bound loop that cannot afford cudaMalloc's
synchronisation); it keeps its partial sums in a fixed array inside the library.  Two calls
in a row must give the same results as each other and as ttc_lqr_bwd_mix, including a shape
whose partial sums do not all fit the array (the variant then runs fewer CTAs).  This file is
named to be collected last, so a run that stops at the first failure has run everything else.
"""
import pytest
import torch

from ttc_cases import solver_inputs_synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import build as ttc_build
    ttc_build.build()
    from ttc_b200 import _lib
    return _lib.load()


def _ptr(t):
    return None if t is None else t.data_ptr()


def _inputs(N, nh, d, rQ, seed):
    A, B, Q, R, _, lA, lB, lQ, h0 = [torch.from_numpy(a).cuda().float() for a in
                                     solver_inputs_synthetic(N, nh, d, d, seed)]
    g = torch.Generator(device="cuda").manual_seed(seed)
    coeff = torch.nn.functional.normalize(torch.rand(N, nh, rQ, device="cuda", generator=g), dim=-1)
    G = torch.randn(rQ, d, d, device="cuda", generator=g) * 0.3
    basis = (G @ G.transpose(1, 2) / d ** 0.5).contiguous()
    du = torch.randn(N, nh, d, device="cuda", generator=g)
    return [A, B, Q, R, coeff, basis, lA, lB, lQ, h0], du


def _grads(xs):
    A, B, Q, R, coeff, basis, lA, lB, lQ, h0 = xs
    return [torch.full_like(t, float("nan")) for t in (A, B, Q, R, coeff, lA, lB, lQ, h0)]


def _check(lib, rc):
    assert rc == 0, lib.ttc_last_error().decode()


@pytest.mark.parametrize("N,nh,d,rQ,T", [(96, 16, 16, 16, 24), (37, 12, 16, 8, 9),
                                        (512, 32, 32, 32, 16)])
def test_noalloc_matches_allocating_backward(lib, N, nh, d, rQ, T):
    xs, du = _inputs(N, nh, d, rQ, seed=N + d)
    A, B, Q, R, coeff, basis, lA, lB, lQ, h0 = xs
    stream = torch.cuda.current_stream().cuda_stream
    u = torch.empty(N, nh, d, device="cuda")
    lam0 = torch.empty(N, nh, d, device="cuda")
    M = torch.empty(N, nh, d, d, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _check(lib, lib.ttc_lqr_fwd_mix(_ptr(A), _ptr(B), _ptr(Q), _ptr(R), _ptr(coeff), _ptr(basis), rQ,
                                    _ptr(lA), _ptr(lB), _ptr(lQ), _ptr(h0), N, nh, d, d, T, 0, 0, _ptr(u),
                                    _ptr(lam0), _ptr(M), _ptr(status), stream))
    common = [_ptr(A), _ptr(B), _ptr(Q), _ptr(R), _ptr(coeff), _ptr(basis), rQ, _ptr(lA), _ptr(lB),
              _ptr(lQ), _ptr(h0), _ptr(lam0), _ptr(M), _ptr(du), N, nh, d, d, T, 0]

    # the allocating entry point: caller-owned slices, summed and symmetrised by the caller
    slices = int(lib.ttc_lqr_bwd_mix_slices(N, nh, d, d, rQ, 0))
    assert slices > 0
    if N == 512:
        # this case is meant to have more partial sums than the library's 16 MiB array holds,
        # so that the variant runs on a capped grid
        assert slices > (4 << 20) // (rQ * d * d), slices
    ref = _grads(xs)
    partial = torch.empty(slices, rQ, d, d, device="cuda")
    gA, gB, gQ, gR, gc, glA, glB, glQ, gh0 = ref
    _check(lib, lib.ttc_lqr_bwd_mix(*common, _ptr(gA), _ptr(gB), _ptr(gQ), _ptr(gR), _ptr(gc),
                                    _ptr(partial), slices, _ptr(glA), _ptr(glB), _ptr(glQ), _ptr(gh0),
                                    _ptr(status), stream))
    S = partial.sum(0)
    ref_basis = 0.5 * (S + S.transpose(-1, -2))

    outs = []
    for _ in range(2):  # two calls in a row share the library's scratch array
        got = _grads(xs)
        gbasis = torch.full((rQ, d, d), float("nan"), device="cuda")
        gA, gB, gQ, gR, gc, glA, glB, glQ, gh0 = got
        _check(lib, lib.ttc_lqr_bwd_mix_noalloc(*common, _ptr(gA), _ptr(gB), _ptr(gQ), _ptr(gR), _ptr(gc),
                                                _ptr(gbasis), _ptr(glA), _ptr(glB), _ptr(glQ), _ptr(gh0),
                                                _ptr(status), stream))
        torch.cuda.synchronize()
        outs.append((got, gbasis))
    assert int(status.item()) == 0
    for got, gbasis in outs:
        # per-row and per-head outputs come from the same kernel code: identical
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
        # the basis gradient sums the same per-CTA partials, possibly over fewer CTAs
        rel = ((gbasis - ref_basis).abs().max() / ref_basis.abs().max()).item()
        assert rel < 1e-5
    for a, b in zip(outs[0][0] + [outs[0][1]], outs[1][0] + [outs[1][1]]):
        assert torch.equal(a, b)


def test_noalloc_rejects_bad_arguments_without_gpu_work(lib):
    from ttc_b200 import _lib
    P = 16  # never dereferenced: rejected before any launch

    def call(d=16, du=16, rQ=8, N=4, grads=P, basis=P):
        return lib.ttc_lqr_bwd_mix_noalloc(*([P] * 6), rQ, *([P] * 4), P, P, P, N, 4, d, du, 8, 0,
                                           *([grads] * 5), basis, *([grads] * 4), P, None)

    assert call(d=64, du=64) == _lib.ERR_UNSUPPORTED
    assert b"h_dim=64" in lib.ttc_last_error()
    assert call(d=32, du=16) == _lib.ERR_UNSUPPORTED
    assert call(rQ=0) == _lib.ERR_INVALID
    assert call(grads=None) == _lib.ERR_INVALID
    # an empty batch with no basis output launches nothing
    assert call(N=0, basis=None) == _lib.OK


def test_noalloc_empty_batch_zeroes_basis_gradient(lib):
    """N = 0: the basis gradient of an empty batch is zero, written into the caller's buffer
    (the allocating path's caller sums zero slices)."""
    rQ, d = 8, 16
    gbasis = torch.full((rQ, d, d), float("nan"), device="cuda")
    P = 16  # per-row pointers: never dereferenced for an empty batch
    rc = lib.ttc_lqr_bwd_mix_noalloc(*([P] * 6), rQ, *([P] * 4), P, P, P, 0, 4, d, d, 8, 0,
                                     *([P] * 5), _ptr(gbasis), *([P] * 4), P,
                                     torch.cuda.current_stream().cuda_stream)
    _check(lib, rc)
    torch.cuda.synchronize()
    assert torch.equal(gbasis, torch.zeros_like(gbasis))
