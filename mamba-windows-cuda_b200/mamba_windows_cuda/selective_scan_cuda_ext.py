"""Checkpoint-level selective scan: drop-in for
mamba_windows_cuda/selective_scan_cuda_ext.py of the reference (:562-677).

``FusedSelectiveScanFunction.apply(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None,
checkpoint_lvl=0) -> (out, h_last)`` and ``FusedSelectiveScan(checkpoint_lvl=0)`` with
``forward`` / ``forward_with_state`` keep the reference's names and arguments:

* ``checkpoint_lvl=0``: the forward saves float32 states every 16 steps (B, L/16, D, 16);
  the backward recomputes the states in between on chip.
* ``checkpoint_lvl=1``: the forward saves only its inputs; the backward first re-runs the
  forward scan to rebuild those checkpoints (less memory, one more forward pass).

Unlike the reference (whose kernels do not compile, and whose backward returned no
gradient for ``h_prev``), the backward returns the ``h_prev`` gradient and honours
``dh_last``.
"""
from __future__ import annotations

import torch

from . import _ops
from .mamba_cuda import _prep


class FusedSelectiveScanFunction(torch.autograd.Function):

    @staticmethod
    def forward(ctx, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None, checkpoint_lvl=0):
        if checkpoint_lvl not in (0, 1):
            raise RuntimeError(f"checkpoint_lvl must be 0 or 1, got {checkpoint_lvl}")
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev = _prep(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
        need = any(ctx.needs_input_grad)
        keep_ckpt = need and checkpoint_lvl == 0
        out, h_last, ckpt, _ = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                               want_h_last=True, want_ckpt=keep_ckpt)
        if need:
            ctx.save_for_backward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, ckpt)
        ctx.checkpoint_lvl = checkpoint_lvl
        ctx.has_h_prev = h_prev is not None
        return out, h_last

    @staticmethod
    def backward(ctx, dout, dh_last):
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, ckpt = ctx.saved_tensors
        if ckpt is None:
            _, _, ckpt, _ = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                            want_out=False, want_ckpt=True)
        dout = dout.contiguous() if dout is not None else None
        dh_last = dh_last.contiguous() if dh_last is not None else None
        du, ddelta, dA, dB, dC, dD, dh_prev = _ops.ss_backward(
            u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, dout, dh_last, ckpt,
            want_dh_prev=ctx.has_h_prev)
        return du, ddelta, dA, dB, dC, dD, dh_prev, None


class FusedSelectiveScan(torch.nn.Module):
    """Selective scan module with a checkpoint level (0: save states, 1: recompute)."""

    def __init__(self, checkpoint_lvl=0):
        super().__init__()
        self.checkpoint_lvl = checkpoint_lvl

    def forward(self, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
        out, _ = FusedSelectiveScanFunction.apply(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                                  self.checkpoint_lvl)
        return out

    def forward_with_state(self, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
        return FusedSelectiveScanFunction.apply(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                                self.checkpoint_lvl)
