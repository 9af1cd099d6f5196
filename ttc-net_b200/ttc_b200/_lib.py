"""ctypes binding of the C-ABI in include/ttc_b200.h (libttc_b200.so, built in-tree).

The library is loaded on first use.  There is no fallback: if it is missing or does
not load, every CUDA entry point raises ``RuntimeError`` naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading

# The in-tree build; TTC_B200_LIB may name another build of the same sources (a variant
# compiled with tuning macros by `build.py --out PATH -D NAME=VALUE`).
LIB_PATH = os.environ.get("TTC_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                          "libttc_b200.so")
ABI_VERSION = 7

DTYPE_F32 = 0
DTYPE_BF16 = 1

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3

STATUS_FWD_UNSTABLE = 1
STATUS_LU_UNSTABLE = 2
STATUS_BWD_UNSTABLE = 4
STATUS_U_NAN = 8
STATUS_MMA_TIMEOUT = 16
STATUS_TRAJ_NONFINITE = 32
STATUS_COPY_TIMEOUT = 64

FLAG_INV_GUARD = 1

# Every symbol include/ttc_b200.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_FP = ctypes.c_void_p      # float* passed as a raw address
_I = ctypes.c_int
_I64 = ctypes.c_int64
SIGNATURES = {
    "ttc_abi_version": (_I, []),
    "ttc_supported": (_I, [_I, _I]),
    "ttc_last_error": (ctypes.c_char_p, []),
    "ttc_lqr_fwd": (_I, [_P] * 9 + [_I64, _I, _I, _I, _I, _I, _I, _P, _FP, _FP, _P, _P]),
    "ttc_lqr_bwd": (_I, [_P] * 9 + [_FP, _FP, _P, _I64, _I, _I, _I, _I, _I, _I] + [_P] * 9 + [_P, _P]),
    "ttc_lqr_rollout": (_I, [_P] * 9 + [_FP, _FP, _P, _I, _I64, _I, _I, _I, _I, _I] + [_P] + [_FP] * 4 + [_P, _P]),
    "ttc_lqr_fwd_affine": (_I, [_P] * 10 + [_I64, _I, _I, _I, _I, _I, _I, _P, _FP, _P, _P]),
    "ttc_lqr_fwd_mix": (_I, [_P] * 6 + [_I] + [_P] * 4 + [_I64, _I, _I, _I, _I, _I, _I, _P, _FP, _FP, _P, _P]),
    "ttc_lqr_bwd_mix_slices": (_I64, [_I64, _I, _I, _I, _I, _I]),
    "ttc_lqr_bwd_mix": (_I, [_P] * 6 + [_I] + [_P] * 4 + [_FP, _FP, _P, _I64, _I, _I, _I, _I, _I]
                        + [_P] * 5 + [_FP, _I64] + [_P] * 4 + [_P, _P]),
    "ttc_lqr_bwd_mix_noalloc": (_I, [_P] * 6 + [_I] + [_P] * 4 + [_FP, _FP, _P, _I64, _I, _I, _I, _I, _I]
                                + [_P] * 5 + [_FP] + [_P] * 4 + [_P, _P]),
    "ttc_lqr_fwd_lowrank": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _I, _P, _P, _P, _P]
                            + [_I64, _I, _I, _I, _I, _I, _I, _P, _FP, _FP, _P, _P]),
    "ttc_lqr_bwd_lowrank": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _I, _P, _P, _P, _P, _FP, _FP, _P]
                            + [_I64, _I, _I, _I, _I, _I] + [_P, _P, _FP, _P, _P, _P, _FP, _I64]
                            + [_P] * 4 + [_P, _P]),
    "ttc_rownorm_fwd": (_I, [_P, _I64, _I, _I, _P, _P]),
    "ttc_rownorm_bwd": (_I, [_P, _P, _I64, _I, _I, _P, _P]),
    "ttc_prologue_fwd": (_I, [_P, _I64] + [_I] * 6 + [_P] * 9 + [_P, _P]),
    "ttc_prologue_bwd": (_I, [_P, _I64] + [_I] * 6 + [_P] * 9 + [_P, _P]),
}

_lib = None
_lock = threading.Lock()


class TTCLibraryError(RuntimeError):
    """The native library is missing, stale or rejected a call."""


def load(path: str | None = None):
    """Load (once) and return the ctypes handle of libttc_b200.so."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise TTCLibraryError(
                f"ttc_b200 CUDA library not found at {p}; build it with "
                "`python ttc-net_b200/build.py` (needs nvcc, targets sm_100a)")
        try:
            lib = ctypes.CDLL(p)
        except OSError as e:  # pragma: no cover - depends on the machine
            raise TTCLibraryError(f"failed to load {p}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        v = lib.ttc_abi_version()
        if v != ABI_VERSION:
            raise TTCLibraryError(f"{p} has ABI version {v}, expected {ABI_VERSION}; rebuild it")
        if path is None:
            _lib = lib
        return lib


def check(rc: int) -> None:
    """Raise for a non-zero return code of a ttc_* call."""
    if rc == OK:
        return
    msg = load().ttc_last_error().decode(errors="replace")
    if rc == ERR_INVALID:
        raise ValueError(f"ttc_b200: {msg}")
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(f"ttc_b200: {msg}")
    raise TTCLibraryError(f"ttc_b200: {msg}")


def supported(d: int, du: int) -> bool:
    return bool(load().ttc_supported(int(d), int(du)))
