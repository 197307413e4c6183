"""Selective scan with grouped B / C:
``selective_scan_grouped(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False)``.

Not in the reference: its B / C are (batch, seqlen, 16), one row per step shared by every
channel. The official Mamba scan also accepts grouped B / C, where each group of channels
has its own rows. Here B, C are (batch, seqlen, G, 16) and channel d reads group
d // (D // G); G = 1 is the reference's layout. Other layouts stay the reference's: u, delta
(batch, seqlen, D), A (D, 16), D (D), h_prev / h_last (batch, D, 16).

Forward and backward run on the GPU (mwc_ss_fwd_grouped / mwc_ss_bwd_grouped). They need
D // G to be a multiple of 128 and the persistent path: 16-byte-aligned buffers, D x element
size a multiple of 16 bytes, and batch x D / 128 at least the SM count or seqlen >= 512.
Other shapes raise RuntimeError.
"""
from __future__ import annotations

import torch

from . import _ops
from .mamba_cuda import selective_scan_ref

__all__ = ["SelectiveScanGroupedFn", "selective_scan_grouped", "selective_scan_grouped_ref"]


def _check(u, delta, A, B, C, D, h_prev):
    for name, t in (("u", u), ("delta", delta), ("A", A), ("B", B), ("C", C), ("D", D)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
        if t.dtype != u.dtype or t.device != u.device:
            raise RuntimeError(f"{name} must match u in dtype and device")
    _ops.dtype_code(u)
    if u.dim() != 3:
        raise RuntimeError("u must be 3D (batch, seqlen, dim)")
    Bb, L, Dd = u.shape
    if B.dim() != 4 or C.dim() != 4 or B.shape != C.shape:
        raise RuntimeError("B and C must be 4D (batch, seqlen, groups, 16) and of one shape")
    G = B.shape[2]
    if tuple(B.shape) != (Bb, L, G, _ops.NSTATE) or G < 1 or Dd % G != 0:
        raise RuntimeError("B / C must be (batch, seqlen, groups, 16) with groups dividing dim")
    if tuple(delta.shape) != (Bb, L, Dd) or tuple(A.shape) != (Dd, _ops.NSTATE) or tuple(D.shape) != (Dd,):
        raise RuntimeError("delta (batch, seqlen, dim), A (dim, 16) and D (dim) shapes required")
    if h_prev is not None and (tuple(h_prev.shape) != (Bb, Dd, _ops.NSTATE) or h_prev.dtype != u.dtype
                               or h_prev.device != u.device):
        raise RuntimeError("h_prev must be (batch, dim, 16) with u's dtype and device")


class SelectiveScanGroupedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, h_prev=None, return_last_state=False):
        ctx.has_D = D is not None
        if D is None:
            D = torch.zeros(u.shape[2], dtype=u.dtype, device=u.device)
        _check(u, delta, A, B, C, D, h_prev)
        u, delta, A, B, C, D = [t.contiguous() for t in (u, delta, A, B, C, D)]
        h_prev = h_prev.contiguous() if h_prev is not None else None
        need = any(ctx.needs_input_grad)
        out, h_last, ckpt, _ = _ops.ss_forward(u, delta, A, B, C, D, h_prev, want_h_last=True,
                                               want_ckpt=need)
        if need:
            ctx.save_for_backward(u, delta, A, B, C, D, h_prev, ckpt)
        ctx.return_last_state = bool(return_last_state)
        return (out, h_last) if return_last_state else out

    @staticmethod
    def backward(ctx, dout, *rest):
        u, delta, A, B, C, D, h_prev, ckpt = ctx.saved_tensors
        dh_last = rest[0] if ctx.return_last_state and rest else None
        dout = dout.contiguous() if dout is not None else None
        dh_last = dh_last.contiguous() if dh_last is not None else None
        du, ddelta, dA, dB, dC, dD, dh_prev = _ops.ss_backward(
            u, delta, A, B, C, D, h_prev, dout, dh_last, ckpt, want_dh_prev=h_prev is not None)
        return du, ddelta, dA, dB, dC, dD if ctx.has_D else None, dh_prev, None


def selective_scan_grouped(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False):
    """Selective scan with grouped B / C (see the module docstring). Returns ``out`` or
    ``(out, h_last)`` with ``return_last_state``."""
    return SelectiveScanGroupedFn.apply(u, delta, A, B, C, D, h_prev, return_last_state)


def selective_scan_grouped_ref(u, delta, A, B, C, D=None, h_prev=None, return_last_state=False):
    """Plain PyTorch version of :func:`selective_scan_grouped` (any device / dtype, autograd):
    the reference's ``selective_scan_ref`` on each group's channels with that group's B / C."""
    G = B.shape[2]
    cpg = u.shape[2] // G
    if D is None:
        D = torch.zeros(u.shape[2], dtype=u.dtype, device=u.device)
    outs, lasts = [], []
    for g in range(G):
        sl = slice(g * cpg, (g + 1) * cpg)
        y, h = selective_scan_ref(u[..., sl], delta[..., sl], A[sl], B[:, :, g], C[:, :, g], D[sl],
                                  h_prev[:, sl] if h_prev is not None else None)
        outs.append(y)
        lasts.append(h)
    out, h_last = torch.cat(outs, dim=2), torch.cat(lasts, dim=1)
    return (out, h_last) if return_last_state else out
