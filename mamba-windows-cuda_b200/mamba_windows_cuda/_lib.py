"""ctypes binding of libmwc_b200.so, the sm_100a C ABI declared in include/mwc_b200.h.

The library is built ahead of time (``make -C mamba-windows-cuda_b200/csrc``); there is
no JIT and no CPU fallback: a missing library raises instead of degrading.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libmwc_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", LIB_NAME)

MWC_F32 = 0
MWC_F16 = 1
MWC_BF16 = 2
MWC_OK = 0
STATUS_NAMES = {1: "invalid argument", 2: "unsupported", 3: "workspace", 4: "CUDA error",
                5: "device wait timed out"}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

# name -> (restype, argtypes); must list every entry point of include/mwc_b200.h
SIGNATURES = {
    "mwc_abi_version": (_int, []),
    "mwc_last_error": (ctypes.c_char_p, []),
    "mwc_build_info": (ctypes.c_char_p, []),
    "mwc_ss_ckpt_count": (_i64, [_i64]),
    "mwc_ss_fwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _int]),
    "mwc_ss_fwd": (_int, [_vp] * 12 + [_i64] * 4 + [_int, _vp]),
    "mwc_ss_bwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _int]),
    "mwc_ss_bwd": (_int, [_vp] * 18 + [_i64] * 4 + [_int, _vp]),
    "mwc_ss_bwd_seq": (_int, [_vp] * 18 + [_i64] * 4 + [_int, _vp]),
    "mwc_ss_adjoint_seq_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "mwc_ss_adjoint_seq": (_int, [_vp] * 7 + [_i64] * 4 + [_int, _vp]),
    "mwc_ss_plan": (_int, [_i64] * 3 + [_int, _int, ctypes.POINTER(ctypes.c_int32)]),
    "mwc_ss_fwd_nstate_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _int]),
    "mwc_ss_fwd_nstate": (_int, [_vp] * 12 + [_i64] * 5 + [_int, _vp]),
    "mwc_ss_fwd_grouped": (_int, [_vp] * 12 + [_i64] * 5 + [_int, _vp]),
    "mwc_ss_bwd_grouped": (_int, [_vp] * 18 + [_i64] * 5 + [_int, _vp]),
    "mwc_ss_fixup": (_int, [_vp] * 8 + [_i64] * 3 + [_int, _vp]),
    "mwc_ss_dprefix_count": (_i64, [_i64]),
    "mwc_ss_fwd_seq": (_int, [_vp] * 13 + [_i64] * 4 + [_int, _vp]),
    "mwc_ss_fixup_chunked": (_int, [_vp] * 9 + [_i64] * 3 + [_int, _vp]),
    "mwc_lin_scan_fwd": (_int, [_vp] * 3 + [_i64] * 3 + [_int, _vp]),
    "mwc_lin_scan_bwd": (_int, [_vp] * 5 + [_i64] * 3 + [_int, _vp]),
    "mwc_ss_fwd_noalloc": (_int, [_vp] * 11 + [_i64] * 3 + [_int, _vp]),
    "mwc_ss_fwd_ex_workspace_bytes": (_i64, [_i64, _i64, _i64, _int]),
    "mwc_ss_fwd_ex": (_int, [_vp] * 8 + [_int] + [_vp] * 6 + [_i64] * 4 + [_int, _vp]),
    "mwc_ss_bwd_ex_workspace_bytes": (_i64, [_i64, _i64, _i64, _int]),
    "mwc_ss_bwd_ex": (_int, [_vp] * 8 + [_int] + [_vp] * 15 + [_i64] * 4 + [_int, _vp]),
    "mwc_conv1d_fwd": (_int, [_vp] * 4 + [_int, _vp] + [_i64] * 4 + [_int, _vp]),
    "mwc_conv1d_bwd_workspace_bytes": (_i64, [_i64] * 4),
    "mwc_conv1d_bwd": (_int, [_vp] * 4 + [_int] + [_vp] * 6 + [_i64] * 5 + [_int, _vp]),
    "mwc_check_last_launch": (_int, [_vp]),
    "mwc_selftest_wait_timeout": (_int, [_vp, _vp]),
}

_lock = threading.Lock()
_lib = None


class LibraryMissing(RuntimeError):
    pass


def load():
    """Load (once) and return the ctypes handle of libmwc_b200.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(
                f"{LIB_NAME} not found at {LIB_PATH}; build it with "
                "`make -C mamba-windows-cuda_b200/csrc` (sm_100a). There is no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.mwc_abi_version() != 1:
            raise LibraryMissing(f"{LIB_NAME} ABI version {lib.mwc_abi_version()} != 1")
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Map a non-zero C-ABI status to RuntimeError (the reference raises RuntimeError
    from TORCH_CHECK for the same conditions)."""
    if rc != MWC_OK:
        msg = load().mwc_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({STATUS_NAMES.get(rc, rc)}): {msg}")
