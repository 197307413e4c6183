"""Float64 composition used as the checker of the extended scan (test infrastructure):
the delta transform and the z gate in numpy around the oracle's scan and its gradients
(the chain rule written out), for selective_scan_fn / mwc_ss_fwd_ex / mwc_ss_bwd_ex."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O


def softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _delta(delta, bias, sp):
    x = delta + bias[None, None, :] if bias is not None else delta
    return x, (softplus(x) if sp else x)


def fwd(u, delta, A, B, C, D, z=None, bias=None, sp=False, h_prev=None):
    """Returns (out, y, h_last): out = y * silu(z) with z, else y."""
    _, de = _delta(delta, bias, sp)
    y, h_last = O.ss_fwd(u, de, A, B, C, D, h_prev)
    out = y * z * sigmoid(z) if z is not None else y
    return out, y, h_last


def bwd(u, delta, A, B, C, D, dout, z=None, bias=None, sp=False, h_prev=None, dh_last=None):
    """Gradients of sum(out * dout) (+ sum(h_last * dh_last)): dict with du, ddelta, dA, dB,
    dC, dD, dh_prev, dbias, dz."""
    x, de = _delta(delta, bias, sp)
    if z is not None:
        y, _ = O.ss_fwd(u, de, A, B, C, D, h_prev)
        s = sigmoid(z)
        gy = dout * z * s
        dz = dout * y * s * (1.0 + z * (1.0 - s))
    else:
        gy, dz = dout, None
    g = O.ss_bwd(u, de, A, B, C, D, gy, h_prev=h_prev, dh_last=dh_last)
    dd = g["ddelta"] * (sigmoid(x) if sp else 1.0)
    g = dict(g)
    g["ddelta"] = dd
    g["dbias"] = dd.sum(axis=(0, 1))
    g["dz"] = dz
    return g
