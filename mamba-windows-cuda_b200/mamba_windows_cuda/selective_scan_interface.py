"""Selective scan with the input / output transforms of Mamba's block, under the official
Mamba argument list: ``selective_scan_fn(u, delta, A, B, C, D=None, z=None,
delta_bias=None, delta_softplus=False, return_last_state=False)``.

The reference (mamba-windows-cuda) has no such entry point: its scans take delta as given
and return the ungated output. Layouts stay the reference's: u, delta, z (B, L, D); B, C
(B, L, 16); A (D, 16); D, delta_bias (D). Semantics:

    delta_eff = softplus(delta + delta_bias)   if delta_softplus, else delta + delta_bias
    y         = selective scan of (u, delta_eff, A, B, C, D)
    out       = y * silu(z)                    when z is given, else y

Forward and backward run on the GPU through mwc_ss_fwd_ex / mwc_ss_bwd_ex; ``h_prev``
(B, D, 16) seeds the state like the reference's stateful scan.
"""
from __future__ import annotations

import torch

from . import _ops
from .mamba_cuda import selective_scan_ref

__all__ = ["SelectiveScanFnEx", "selective_scan_fn", "selective_scan_ref_ex"]


class SelectiveScanFnEx(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                return_last_state=False, h_prev=None):
        ctx.has_D = D is not None
        if D is None:
            D = torch.zeros(u.shape[2], dtype=u.dtype, device=u.device)
        _ops.check_ss_inputs(u, delta, A, B, C, D, h_prev)
        if z is not None and (not isinstance(z, torch.Tensor) or z.shape != u.shape or z.dtype != u.dtype
                              or z.device != u.device):
            raise RuntimeError("z must match u in shape, dtype and device")
        if delta_bias is not None and (not isinstance(delta_bias, torch.Tensor) or delta_bias.shape != (u.shape[2],)
                                       or delta_bias.dtype != u.dtype or delta_bias.device != u.device):
            raise RuntimeError("delta_bias must be (D,) with u's dtype and device")
        u, delta, A, B, C, D = [t.contiguous() for t in (u, delta, A, B, C, D)]
        z = z.contiguous() if z is not None else None
        delta_bias = delta_bias.contiguous() if delta_bias is not None else None
        h_prev = h_prev.contiguous() if h_prev is not None else None
        need = any(ctx.needs_input_grad)
        out, out_z, h_last, ckpt = _ops.ss_forward_ex(
            u, delta, A, B, C, D, z, delta_bias, delta_softplus, h_prev,
            want_h_last=True, want_ckpt=need)
        if need:
            ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, h_prev, out, ckpt)
        ctx.delta_softplus = bool(delta_softplus)
        ctx.return_last_state = bool(return_last_state)
        result = out_z if z is not None else out
        if return_last_state:
            return result, h_last
        return result

    @staticmethod
    def backward(ctx, dout, *rest):
        u, delta, A, B, C, D, z, delta_bias, h_prev, out, ckpt = ctx.saved_tensors
        dh_last = rest[0] if ctx.return_last_state and rest else None
        dout = dout.contiguous() if dout is not None else None
        dh_last = dh_last.contiguous() if dh_last is not None else None
        du, ddelta, dA, dB, dC, dD, dbias, dz, dh_prev = _ops.ss_backward_ex(
            u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus, h_prev, out, dout, dh_last,
            ckpt, want_dbias=delta_bias is not None, want_dh_prev=h_prev is not None)
        return du, ddelta, dA, dB, dC, dD if ctx.has_D else None, dz, dbias, None, None, dh_prev


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                      return_last_state=False, h_prev=None):
    """Selective scan with delta bias / softplus and the z gate (see the module docstring).
    Returns ``out`` or ``(out, h_last)`` with ``return_last_state``."""
    return SelectiveScanFnEx.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                                   return_last_state, h_prev)


def selective_scan_ref_ex(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                          return_last_state=False, h_prev=None):
    """Plain PyTorch version of :func:`selective_scan_fn` (any device / dtype, autograd):
    the transforms in PyTorch around the reference's ``selective_scan_ref``."""
    if D is None:
        D = torch.zeros(u.shape[2], dtype=u.dtype, device=u.device)
    dl = delta + delta_bias if delta_bias is not None else delta
    if delta_softplus:
        dl = torch.nn.functional.softplus(dl)
    y, h_last = selective_scan_ref(u, dl, A, B, C, D, h_prev)
    out = y * torch.nn.functional.silu(z) if z is not None else y
    return (out, h_last) if return_last_state else out
