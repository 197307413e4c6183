"""Selective scan with N = 16, 32 or 64 states per channel:
``selective_scan_nstate(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False)``
(forward and backward) and ``selective_scan_forward_nstate`` (forward only, one kernel).

Not in the reference: it supports N = 16 only and rejects other state sizes
(mamba_cuda.py:186-238); the official Mamba scan takes larger N. The state size comes from A
(D, N); B, C are (batch, seqlen, N), h_prev / h_last (batch, D, N); u, delta (batch, seqlen,
D) as in the reference. N = 16 runs the regular forward (mwc_ss_fwd); N = 32 / 64 run the
generic forward kernels through mwc_ss_fwd_nstate.

selective_scan_forward_nstate is forward only (inputs that require gradients raise
RuntimeError while gradient recording is on). selective_scan_nstate has gradients: the
recurrence is independent per state, so an N-state scan is N / 16 scans of 16-state slices
on the regular 16-state kernels. The slices couple only through sums: the output adds their
<C, h> terms (D u counted once, in slice 0), du and ddelta add theirs, and dD comes from
slice 0; h_last, dA, dB, dC and dh_prev are the slices' results side by side.
"""
from __future__ import annotations

import torch

from . import _ops

__all__ = ["SelectiveScanNStateFn", "selective_scan_forward_nstate", "selective_scan_nstate"]

SUPPORTED_N = (16, 32, 64)


def _check(u, delta, A, B, C, D, h_prev):
    tensors = (u, delta, A, B, C, D) + ((h_prev,) if h_prev is not None else ())
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("inputs must be CUDA tensors")
        if t.dtype != u.dtype or t.device != u.device:
            raise RuntimeError("inputs must match u in dtype and device")
    _ops.dtype_code(u)
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
    return N


class SelectiveScanNStateFn(torch.autograd.Function):
    """N = 16 / 32 / 64 as N / 16 state slices on the 16-state kernels (see the module docstring)."""

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, h_prev=None, return_last_state=False):
        ctx.has_D = D is not None
        if D is None:
            D = torch.zeros(u.shape[2], dtype=u.dtype, device=u.device)
        N = _check(u, delta, A, B, C, D, h_prev)
        u, delta = u.contiguous(), delta.contiguous()
        zeroD = torch.zeros_like(D)
        need = any(ctx.needs_input_grad)
        slices, outs, lasts = [], [], []
        for j in range(N // _ops.NSTATE):
            sl = slice(j * _ops.NSTATE, (j + 1) * _ops.NSTATE)
            Aj, Bj, Cj = A[:, sl].contiguous(), B[..., sl].contiguous(), C[..., sl].contiguous()
            Dj = D.contiguous() if j == 0 else zeroD
            hj = h_prev[..., sl].contiguous() if h_prev is not None else None
            out, h_last, ckpt, _ = _ops.ss_forward(u, delta, Aj, Bj, Cj, Dj, hj, want_h_last=True,
                                                   want_ckpt=need)
            outs.append(out)
            lasts.append(h_last)
            slices.append((Aj, Bj, Cj, Dj, hj, ckpt))
        out = outs[0]
        for o in outs[1:]:
            out = out + o
        if need:
            ctx.save_for_backward(u, delta, *[t for s in slices for t in s])
        ctx.nslices = len(slices)
        ctx.has_h_prev = h_prev is not None
        ctx.return_last_state = bool(return_last_state)
        h_last = torch.cat(lasts, dim=2)
        return (out, h_last) if return_last_state else out

    @staticmethod
    def backward(ctx, dout, *rest):
        saved = ctx.saved_tensors
        u, delta = saved[0], saved[1]
        dh_last = rest[0] if ctx.return_last_state and rest else None
        dout = dout.contiguous() if dout is not None else None
        du = ddelta = dD = None
        dAs, dBs, dCs, dhps = [], [], [], []
        for j in range(ctx.nslices):
            Aj, Bj, Cj, Dj, hj, ckpt = saved[2 + 6 * j: 8 + 6 * j]
            sl = slice(j * _ops.NSTATE, (j + 1) * _ops.NSTATE)
            dhl = dh_last[..., sl].contiguous() if dh_last is not None else None
            g = _ops.ss_backward(u, delta, Aj, Bj, Cj, Dj, hj, dout, dhl, ckpt,
                                 want_dh_prev=ctx.has_h_prev)
            du = g[0] if du is None else du + g[0]
            ddelta = g[1] if ddelta is None else ddelta + g[1]
            dAs.append(g[2])
            dBs.append(g[3])
            dCs.append(g[4])
            if j == 0:
                dD = g[5]
            dhps.append(g[6])
        dh_prev = torch.cat(dhps, dim=2) if ctx.has_h_prev else None
        return (du, ddelta, torch.cat(dAs, dim=1), torch.cat(dBs, dim=2), torch.cat(dCs, dim=2),
                dD if ctx.has_D else None, dh_prev, None)


def selective_scan_nstate(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False):
    """Selective scan with N = 16, 32 or 64 states and gradients (see the module docstring).
    Returns ``out`` or ``(out, h_last)`` with ``return_last_state``."""
    return SelectiveScanNStateFn.apply(u, delta, A, B, C, D, h_prev, return_last_state)


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
