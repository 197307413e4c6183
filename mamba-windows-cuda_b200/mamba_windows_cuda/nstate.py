"""Forward selective scan with N = 16, 32 or 64 states per channel:
``selective_scan_forward_nstate(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False)``.

Not in the reference: it supports N = 16 only and rejects other state sizes
(mamba_cuda.py:186-238); the official Mamba scan takes larger N. The state size comes from A
(D, N); B, C are (batch, seqlen, N), h_prev / h_last (batch, D, N); u, delta (batch, seqlen,
D) as in the reference. N = 16 runs the regular forward (mwc_ss_fwd); N = 32 / 64 run the
generic forward kernels through mwc_ss_fwd_nstate.

Forward only: there is no backward for N = 32 / 64 here, so inputs that require gradients
raise RuntimeError while gradient recording is on (wrap inference in torch.no_grad()).
"""
from __future__ import annotations

import torch

from . import _ops

__all__ = ["selective_scan_forward_nstate"]

SUPPORTED_N = (16, 32, 64)


def selective_scan_forward_nstate(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False):
    """Forward scan with N states per channel (see the module docstring). Returns ``out`` or
    ``(out, h_last)`` with ``return_last_state``."""
    if D is None:
        D = torch.zeros(u.shape[2], dtype=u.dtype, device=u.device)
    tensors = (u, delta, A, B, C, D) + ((h_prev,) if h_prev is not None else ())
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("inputs must be CUDA tensors")
        if t.dtype != u.dtype or t.device != u.device:
            raise RuntimeError("inputs must match u in dtype and device")
    _ops.dtype_code(u)
    if torch.is_grad_enabled() and any(t.requires_grad for t in tensors):
        raise RuntimeError("selective_scan_forward_nstate is forward only (no backward for N = 32 / 64)")
    if u.dim() != 3 or A.dim() != 2:
        raise RuntimeError("u must be (batch, seqlen, dim) and A (dim, N)")
    Bb, L, Dd = u.shape
    N = A.shape[1]
    if N not in SUPPORTED_N:
        raise RuntimeError(f"N must be one of {SUPPORTED_N} (got {N})")
    if (tuple(delta.shape) != (Bb, L, Dd) or tuple(A.shape) != (Dd, N) or tuple(B.shape) != (Bb, L, N)
            or tuple(C.shape) != (Bb, L, N) or tuple(D.shape) != (Dd,)):
        raise RuntimeError("shapes: delta (batch, seqlen, dim), A (dim, N), B / C (batch, seqlen, N), D (dim)")
    if h_prev is not None and tuple(h_prev.shape) != (Bb, Dd, N):
        raise RuntimeError("h_prev must be (batch, dim, N)")
    args = [t.contiguous() for t in (u, delta, A, B, C, D)]
    h_prev = h_prev.contiguous() if h_prev is not None else None
    out, h_last, _, _ = _ops.ss_forward(*args, h_prev, want_h_last=return_last_state)
    return (out, h_last) if return_last_state else out
