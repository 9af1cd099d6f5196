"""CPU checks of the C-ABI library: it builds for sm_100a, loads, exports every symbol
include/ttc_b200.h declares, and rejects bad arguments before touching the GPU."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "ttc_b200.h")


@pytest.fixture(scope="module")
def lib():
    import build as ttc_build  # ttc-net_b200/build.py
    from ttc_b200 import _lib
    ttc_build.build()
    return _lib.load()


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ttc_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("ttc_lqr_fwd", "ttc_lqr_bwd", "ttc_lqr_rollout", "ttc_prologue_fwd", "ttc_prologue_bwd",
              "ttc_abi_version", "ttc_supported", "ttc_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from ttc_b200 import _lib
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ttc_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version(lib):
    from ttc_b200 import _lib
    assert lib.ttc_abi_version() == _lib.ABI_VERSION


def test_supported_shapes(lib):
    assert lib.ttc_supported(16, 16) == 1
    assert lib.ttc_supported(32, 32) == 1
    assert lib.ttc_supported(64, 64) == 1
    assert lib.ttc_supported(24, 24) == 0
    assert lib.ttc_supported(32, 16) == 1   # u_dim < h_dim, multiples of 16
    assert lib.ttc_supported(64, 32) == 1
    assert lib.ttc_supported(64, 16) == 1
    assert lib.ttc_supported(16, 32) == 0   # u_dim > h_dim
    assert lib.ttc_supported(32, 8) == 0    # u_dim not a multiple of 16


def _fwd(lib, N=1, nh=1, d=16, du=16, T=4, dtype=0, null_inputs=False, flags=0):
    p = None if null_inputs else 16  # never dereferenced: rejected before any launch
    return lib.ttc_lqr_fwd(*([p] * 9), N, nh, d, du, T, dtype, flags, p, p, None, p, None)


def test_fwd_rejects_bad_arguments_without_gpu(lib):
    from ttc_b200 import _lib
    assert _fwd(lib, N=-1) == _lib.ERR_INVALID
    assert b"N (rows)" in lib.ttc_last_error()
    assert _fwd(lib, nh=0) == _lib.ERR_INVALID
    assert _fwd(lib, T=0) == _lib.ERR_INVALID
    assert _fwd(lib, dtype=7) == _lib.ERR_INVALID
    assert _fwd(lib, d=24, du=24) == _lib.ERR_UNSUPPORTED
    assert b"h_dim=24" in lib.ttc_last_error()
    assert _fwd(lib, null_inputs=True) == _lib.ERR_INVALID
    assert _fwd(lib, flags=6) == _lib.ERR_INVALID
    assert b"flag" in lib.ttc_last_error()
    assert _fwd(lib, N=0) == _lib.OK  # empty batch: nothing to launch


def test_bwd_rejects_bad_arguments_without_gpu(lib):
    from ttc_b200 import _lib
    P = 16
    base = dict(N=1, nh=1, d=16, du=16, T=4, dtype=0)

    def bwd(Qf=P, lam0=P, M=P, grads=P, **kw):
        a = {**base, **kw}
        return lib.ttc_lqr_bwd(P, P, P, P, Qf, P, P, P, P, lam0, M, P, a["N"], a["nh"], a["d"],
                               a["du"], a["T"], a["dtype"], 0, *([grads] * 9), P, None)

    assert bwd(M=None, Qf=None) == _lib.ERR_INVALID        # recompute needs Q_f
    assert bwd(lam0=None) == _lib.ERR_INVALID              # M without lam0
    assert bwd(grads=None) == _lib.ERR_INVALID
    assert bwd(d=48, du=48) == _lib.ERR_UNSUPPORTED
    assert bwd(N=0) == _lib.OK


def test_prologue_rejects_bad_arguments_without_gpu(lib):
    from ttc_b200 import _lib
    P = 16  # never dereferenced: rejected before any launch

    def fwd(N=1, nh=1, d=16, du=16, rB=16, rQ=16, dtype=0, outs=P):
        return lib.ttc_prologue_fwd(P, N, nh, d, du, rB, rQ, dtype, *([outs] * 9), None, None)

    def bwd(N=1, nh=1, d=16, du=16, rB=16, rQ=16, dtype=0, dZ=P):
        return lib.ttc_prologue_bwd(P, N, nh, d, du, rB, rQ, dtype, *([None] * 9), dZ, None)

    assert fwd(N=-1) == _lib.ERR_INVALID
    assert fwd(nh=0) == _lib.ERR_INVALID
    assert fwd(rB=0) == _lib.ERR_INVALID
    assert fwd(dtype=5) == _lib.ERR_INVALID
    assert fwd(d=65) == _lib.ERR_UNSUPPORTED
    assert b"<= 64" in lib.ttc_last_error()
    assert fwd(outs=None) == _lib.ERR_INVALID
    assert fwd(N=0) == _lib.OK
    assert bwd(dZ=None) == _lib.ERR_INVALID
    assert bwd(rQ=100) == _lib.ERR_UNSUPPORTED
    assert bwd(N=0) == _lib.OK


def test_rollout_rejects_bad_arguments_without_gpu(lib):
    from ttc_b200 import _lib
    P = 16  # never dereferenced: rejected before any launch

    def roll(Qf=P, lam0=P, M=P, r0=None, u=P, cost=None, N=1, nh=1, d=16, du=16, T=4, dtype=0, r_steps=1):
        return lib.ttc_lqr_rollout(P, P, P, P, Qf, P, P, P, P, lam0, M, r0, r_steps, N, nh, d, du, T, dtype,
                                   u, None, None, None, cost, P, None)

    assert roll(N=-1) == _lib.ERR_INVALID
    assert roll(T=0) == _lib.ERR_INVALID
    assert roll(d=16, du=32) == _lib.ERR_UNSUPPORTED
    assert roll(lam0=None) == _lib.ERR_INVALID
    assert roll(u=None) == _lib.ERR_INVALID
    assert roll(r0=P, M=None) == _lib.ERR_INVALID          # affine term needs M
    assert b"r0" in lib.ttc_last_error()
    assert roll(cost=P, Qf=None) == _lib.ERR_INVALID       # cost needs Q_f
    assert roll(N=1 << 20, nh=64, T=64) == _lib.ERR_INVALID  # N * nh * T >= 2^31
    assert roll(N=0) == _lib.OK
    assert roll(r_steps=2) == _lib.ERR_INVALID             # r_steps is 1 or T
    assert roll(r0=P, r_steps=4) == _lib.ERR_INVALID       # every-step affine term: no M
    assert b"ttc_lqr_fwd_affine" in lib.ttc_last_error()


def test_affine_forward_rejects_bad_arguments_without_gpu(lib):
    from ttc_b200 import _lib
    P = 16

    def fwd(r=P, lam0=P, N=1, nh=1, d=16, du=16, T=4, dtype=0, flags=0):
        return lib.ttc_lqr_fwd_affine(P, P, P, P, P, P, P, P, P, r, N, nh, d, du, T, dtype, flags, P, lam0, P,
                                      None)

    assert fwd(N=-1) == _lib.ERR_INVALID
    assert fwd(T=0) == _lib.ERR_INVALID
    assert fwd(d=16, du=32) == _lib.ERR_UNSUPPORTED
    assert fwd(r=None) == _lib.ERR_INVALID
    assert fwd(lam0=None) == _lib.ERR_INVALID
    assert fwd(flags=8) == _lib.ERR_INVALID
    assert fwd(N=1 << 20, nh=64, T=64) == _lib.ERR_INVALID
    assert fwd(N=0) == _lib.OK
