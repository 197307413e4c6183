"""CPU oracle for the selective scan and the linear-recurrence scan.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline / reference leg of ``bench.py`` may import this module. The product path
(``mamba_windows_cuda``) never imports it and has no CPU fallback.

Two restatements of the reference algorithm live here:

* ``ss_fwd`` / ``ss_bwd`` / ``lin_fwd`` / ``lin_bwd`` call ``liboracle_scan.so``
  (``scan_oracle.c``): float64, OpenMP over channels, any size.
* ``np_ss_fwd`` / ``np_ss_bwd`` are a plain numpy restatement (Python loop over time),
  used only on small cases to cross-check the C code.

Both follow ``mamba_windows_cuda/mamba_cuda.py:875-946`` (``selective_scan_ref`` with the
time axis of the einsum at :910 placed last) and ``pscan.py:153-171``
(``parallel_scan_ref``). Their agreement with the reference's own Python code is pinned
by ``tests/test_oracle.py`` against the fixtures in ``tests/golden``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_scan.so")
_lib = None

_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64


def build() -> str:
    """Compile liboracle_scan.so with the Makefile next to this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    lib.orc_num_threads.restype = ctypes.c_int
    lib.orc_set_threads.argtypes = [ctypes.c_int]
    lib.orc_ss_fwd.argtypes = [_f64p] * 9 + [_i64] * 4 + [ctypes.c_int]
    lib.orc_ss_bwd.argtypes = [_f64p] * 16 + [_i64] * 4 + [ctypes.c_int]
    lib.orc_lin_fwd.argtypes = [_f64p] * 3 + [_i64] * 3
    lib.orc_lin_bwd.argtypes = [_f64p] * 5 + [_i64] * 3
    _lib = lib
    return lib


def set_threads(n: int) -> None:
    _load().orc_set_threads(int(n))


def num_threads() -> int:
    return int(_load().orc_num_threads())


def _c(x):
    """float64, C-contiguous copy (or view) of an array-like; None stays None."""
    if x is None:
        return None
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().cpu().double().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float64))


def _p(x):
    if x is None:
        return ctypes.cast(None, _f64p)
    return x.ctypes.data_as(_f64p)


def ss_fwd(u, delta, A, Bm, Cm, Dv, h_prev=None, clamp=True):
    """Forward selective scan in float64. Returns (out (B,L,D), h_last (B,D,N))."""
    lib = _load()
    u, delta, A, Bm, Cm, Dv, h_prev = map(_c, (u, delta, A, Bm, Cm, Dv, h_prev))
    B, L, D = u.shape
    N = A.shape[1]
    out = np.empty((B, L, D))
    h_last = np.empty((B, D, N))
    lib.orc_ss_fwd(_p(u), _p(delta), _p(A), _p(Bm), _p(Cm), _p(Dv), _p(h_prev),
                   _p(out), _p(h_last), B, L, D, N, int(bool(clamp)))
    return out, h_last


def ss_bwd(u, delta, A, Bm, Cm, Dv, dout, h_prev=None, dh_last=None, clamp=True):
    """Gradients of sum(out*dout) + sum(h_last*dh_last) in float64.

    Returns a dict with du, ddelta, dA, dB, dC, dD and dh_prev.
    """
    lib = _load()
    u, delta, A, Bm, Cm, Dv, dout, h_prev, dh_last = map(
        _c, (u, delta, A, Bm, Cm, Dv, dout, h_prev, dh_last))
    B, L, D = u.shape
    N = A.shape[1]
    g = {
        "du": np.empty((B, L, D)), "ddelta": np.empty((B, L, D)),
        "dA": np.empty((D, N)), "dB": np.empty((B, L, N)), "dC": np.empty((B, L, N)),
        "dD": np.empty((D,)), "dh_prev": np.empty((B, D, N)),
    }
    lib.orc_ss_bwd(_p(u), _p(delta), _p(A), _p(Bm), _p(Cm), _p(Dv), _p(h_prev),
                   _p(dout), _p(dh_last), _p(g["du"]), _p(g["ddelta"]), _p(g["dA"]),
                   _p(g["dB"]), _p(g["dC"]), _p(g["dD"]), _p(g["dh_prev"]),
                   B, L, D, N, int(bool(clamp)))
    return g


def lin_fwd(a, x):
    """H_0 = X_0, H_t = A_t H_{t-1} + X_t along axis 2 of (B, D, L, N); float64."""
    lib = _load()
    a, x = _c(a), _c(x)
    shape = x.shape
    Bb, Dd, L, N = shape
    h = np.empty(shape)
    lib.orc_lin_fwd(_p(a), _p(x), _p(h), Bb * Dd, L, N)
    return h


def lin_bwd(a, h, g):
    """(gA, gX) of sum(H * g) for lin_fwd; float64."""
    lib = _load()
    a, h, g = _c(a), _c(h), _c(g)
    Bb, Dd, L, N = g.shape
    ga = np.empty(g.shape)
    gx = np.empty(g.shape)
    lib.orc_lin_bwd(_p(a), _p(h), _p(g), _p(ga), _p(gx), Bb * Dd, L, N)
    return ga, gx


# ---------------------------------------------------------------------------
# numpy restatement (small cases only): vectorised over (b, d, n), loop over t
# ---------------------------------------------------------------------------

def np_ss_fwd(u, delta, A, Bm, Cm, Dv, h_prev=None):
    u, delta, A, Bm, Cm, Dv, h_prev = map(_c, (u, delta, A, Bm, Cm, Dv, h_prev))
    B, L, D = u.shape
    N = A.shape[1]
    h = np.zeros((B, D, N)) if h_prev is None else h_prev.copy()
    out = np.empty((B, L, D))
    for t in range(L):
        a = np.exp(delta[:, t, :, None] * A[None])
        h = a * h + (delta[:, t, :] * u[:, t, :])[:, :, None] * Bm[:, t, None, :]
        out[:, t, :] = np.einsum("bdn,bn->bd", h, Cm[:, t, :]) + Dv[None] * u[:, t, :]
    return out, h


def np_ss_bwd(u, delta, A, Bm, Cm, Dv, dout, h_prev=None, dh_last=None):
    u, delta, A, Bm, Cm, Dv, dout, h_prev, dh_last = map(
        _c, (u, delta, A, Bm, Cm, Dv, dout, h_prev, dh_last))
    B, L, D = u.shape
    N = A.shape[1]
    hs = np.empty((L + 1, B, D, N))
    hs[0] = 0.0 if h_prev is None else h_prev
    for t in range(L):
        a = np.exp(delta[:, t, :, None] * A[None])
        hs[t + 1] = a * hs[t] + (delta[:, t, :] * u[:, t, :])[:, :, None] * Bm[:, t, None, :]
    q = np.zeros((B, D, N)) if dh_last is None else dh_last.copy()
    du = np.empty((B, L, D)); ddelta = np.empty((B, L, D))
    dA = np.zeros((D, N)); dB = np.empty((B, L, N)); dC = np.empty((B, L, N))
    for t in range(L - 1, -1, -1):
        dt, uu, gy = delta[:, t, :], u[:, t, :], dout[:, t, :]
        a = np.exp(dt[:, :, None] * A[None])
        g = gy[:, :, None] * Cm[:, t, None, :] + q
        ah = a * hs[t]
        dC[:, t, :] = np.einsum("bd,bdn->bn", gy, hs[t + 1])
        dB[:, t, :] = np.einsum("bdn,bd->bn", g, dt * uu)
        sgb = np.einsum("bdn,bn->bd", g, Bm[:, t, :])
        du[:, t, :] = gy * Dv[None] + dt * sgb
        ddelta[:, t, :] = np.einsum("bdn,dn->bd", g * ah, A) + uu * sgb
        dA += np.einsum("bdn,bd->dn", g * ah, dt)
        q = a * g
    dD = np.einsum("bld,bld->d", dout, u)
    return {"du": du, "ddelta": ddelta, "dA": dA, "dB": dB, "dC": dC, "dD": dD,
            "dh_prev": q}
