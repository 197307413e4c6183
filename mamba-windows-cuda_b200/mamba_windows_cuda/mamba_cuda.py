"""Selective scan (N = 16): drop-in for mamba_windows_cuda/mamba_cuda.py of the reference.

Public surface kept from the reference (same names, arguments, returns and errors):

* ``SelectiveScanCuda`` (mamba_cuda.py:1172-1219): zero-argument ``nn.Module`` with
  ``forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None) -> out`` and
  ``forward_with_state(...) -> (out, h_last)``.
* ``SelectiveScanFnV2`` (:1136-1169, the default training path), ``SelectiveScanFn``
  (:1099-1133, recompute variant) and ``SelectiveScanCudaFunction`` (:1044-1096, stateful
  ``h_prev`` / ``h_last`` path) autograd Functions.
* ``selective_scan_ref`` (:875-946) and ``selective_scan_backward`` (:949-1041): plain
  PyTorch restatements kept as API (the reference's test suite imports the former).

Every CUDA path runs the sm_100a kernels of libmwc_b200.so: the forward scan writes
float32 checkpoints every 16 steps, the backward is a reverse-scan kernel that recomputes
states from them (also for the stateful ``h_prev`` path, where the reference fell back to
a Python loop). There is no CPU fallback: CPU tensors raise like the reference's
TORCH_CHECK(u.is_cuda()).
"""
from __future__ import annotations

import torch

from . import _ops


def _prep(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
    _ops.check_ss_inputs(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
    c = [t.contiguous() for t in (u, delta, A, B_ssm, C_ssm, D_ssm)]
    return c + [h_prev.contiguous() if h_prev is not None else None]


class _SelectiveScanOps:
    """The op module the reference JIT-built (``_get_selective_scan_cuda_module``,
    mamba_cuda.py:835-872), with its five entry points (declarations at :793-830), backed by
    libmwc_b200.so. Arguments, return values and RuntimeError validation follow the
    reference host functions. One difference in kind: the reference's ``h_bank`` (every
    state, (B, D, L, 16) in the input dtype) is here the float32 checkpoint tensor
    (B, ceil(L / 16), D, 16), the state after every 16th step, from which
    ``selective_scan_cuda_backward_direct`` recomputes the rest; pass it through unchanged."""

    @staticmethod
    def selective_scan_cuda_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev_opt=None):
        """mamba_cuda.py:176-269: ``out`` (B, L, D), starting from ``h_prev_opt`` (or 0)."""
        args = _prep(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev_opt)
        return _ops.ss_forward(*args)[0]

    @staticmethod
    def selective_scan_cuda_forward_with_state(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev_opt=None):
        """mamba_cuda.py:271-359: ``[out, h_last]``."""
        args = _prep(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev_opt)
        out, h_last, _, _ = _ops.ss_forward(*args, want_h_last=True)
        return [out, h_last]

    @staticmethod
    def selective_scan_cuda_backward(u, delta, A, B_ssm, C_ssm, D_ssm, grad_out):
        """mamba_cuda.py:564-604 (recompute backward, h0 = 0): rebuilds the checkpoints with
        a forward pass, then runs the reverse scan. Returns ``[du, ddelta, dA, dB, dC, dD]``."""
        args = _prep(u, delta, A, B_ssm, C_ssm, D_ssm)[:6]
        _, _, ckpt, _ = _ops.ss_forward(*args, want_out=False, want_ckpt=True)
        return list(_ops.ss_backward(*args, None, grad_out.contiguous(), None, ckpt)[:6])

    @staticmethod
    def selective_scan_cuda_forward_store(u, delta, A, B_ssm, C_ssm, D_ssm):
        """mamba_cuda.py:747-764: ``[out, h_bank]`` with h0 = 0 (h_bank: float32
        checkpoints, see the class docstring)."""
        args = _prep(u, delta, A, B_ssm, C_ssm, D_ssm)[:6]
        out, _, ckpt, _ = _ops.ss_forward(*args, want_ckpt=True)
        return [out, ckpt]

    @staticmethod
    def selective_scan_cuda_backward_direct(u, delta, A, B_ssm, C_ssm, D_ssm, grad_out, h_bank):
        """mamba_cuda.py:766-790: ``[du, ddelta, dA, dB, dC, dD]`` from the states that
        ``selective_scan_cuda_forward_store`` returned."""
        args = _prep(u, delta, A, B_ssm, C_ssm, D_ssm)[:6]
        Bb, L, D = args[0].shape
        if (not isinstance(h_bank, torch.Tensor) or h_bank.dtype != torch.float32
                or tuple(h_bank.shape) != (Bb, _ops.ckpt_count(L), D, _ops.NSTATE)):
            raise RuntimeError("h_bank must be the float32 (B, ceil(L/16), D, 16) states that "
                               "selective_scan_cuda_forward_store returned")
        return list(_ops.ss_backward(*args, None, grad_out.contiguous(), None,
                                     h_bank.contiguous())[:6])


_selective_scan_cuda_module = None


def _get_selective_scan_cuda_module():
    """The op module with the reference's five entry points (mamba_cuda.py:835-872). The
    reference JIT-compiled it here; this build loads the prebuilt sm_100a library instead
    and raises if it is missing (there is no CPU fallback)."""
    global _selective_scan_cuda_module
    if _selective_scan_cuda_module is None:
        from . import _lib
        _lib.load()
        _selective_scan_cuda_module = _SelectiveScanOps()
    return _selective_scan_cuda_module


class SelectiveScanCudaFunction(torch.autograd.Function):
    """Stateful selective scan: ``(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None) ->
    (out, h_last)``. Gradients flow to all inputs, ``h_prev`` included, through the CUDA
    reverse-scan kernel (``dh_last`` is honoured)."""

    @staticmethod
    def forward(ctx, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev = _prep(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
        need = any(ctx.needs_input_grad)
        out, h_last, ckpt, _ = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                               want_h_last=True, want_ckpt=need)
        if need:
            ctx.save_for_backward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, ckpt)
        ctx.has_h_prev = h_prev is not None
        return out, h_last

    @staticmethod
    def backward(ctx, dout, dh_last):
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, ckpt = ctx.saved_tensors
        dout = dout.contiguous() if dout is not None else None
        dh_last = dh_last.contiguous() if dh_last is not None else None
        du, ddelta, dA, dB, dC, dD, dh_prev = _ops.ss_backward(
            u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, dout, dh_last, ckpt,
            want_dh_prev=ctx.has_h_prev)
        return du, ddelta, dA, dB, dC, dD, dh_prev


class SelectiveScanFn(torch.autograd.Function):
    """Recompute variant (reference V1, mamba_cuda.py:1099-1133): the forward keeps only
    the inputs; the backward first re-runs the forward scan to rebuild the float32
    checkpoints, then runs the reverse scan."""

    @staticmethod
    def _get_module():
        return _get_selective_scan_cuda_module()

    @staticmethod
    def forward(ctx, u, delta, A, B_ssm, C_ssm, D_ssm):
        u, delta, A, B_ssm, C_ssm, D_ssm, _ = _prep(u, delta, A, B_ssm, C_ssm, D_ssm)
        out, _, _, _ = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm)
        ctx.save_for_backward(u, delta, A, B_ssm, C_ssm, D_ssm)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        u, delta, A, B_ssm, C_ssm, D_ssm = ctx.saved_tensors
        _, _, ckpt, _ = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, want_out=False,
                                        want_ckpt=True)
        du, ddelta, dA, dB, dC, dD, _ = _ops.ss_backward(
            u, delta, A, B_ssm, C_ssm, D_ssm, None, grad_out.contiguous(), None, ckpt)
        return du, ddelta, dA, dB, dC, dD


class SelectiveScanFnV2(torch.autograd.Function):
    """Default training path (reference V2, mamba_cuda.py:1136-1169). The reference's
    forward stored every state (a (B, D, L, 16) bank); here the forward stores one float32
    state per 16 steps and the backward recomputes the rest in registers."""

    @staticmethod
    def _get_module():
        return _get_selective_scan_cuda_module()

    @staticmethod
    def forward(ctx, u, delta, A, B_ssm, C_ssm, D_ssm):
        u, delta, A, B_ssm, C_ssm, D_ssm, _ = _prep(u, delta, A, B_ssm, C_ssm, D_ssm)
        need = any(ctx.needs_input_grad)
        out, _, ckpt, _ = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, want_ckpt=need)
        if need:
            ctx.save_for_backward(u, delta, A, B_ssm, C_ssm, D_ssm, ckpt)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        u, delta, A, B_ssm, C_ssm, D_ssm, ckpt = ctx.saved_tensors
        du, ddelta, dA, dB, dC, dD, _ = _ops.ss_backward(
            u, delta, A, B_ssm, C_ssm, D_ssm, None, grad_out.contiguous(), None, ckpt)
        return du, ddelta, dA, dB, dC, dD


class SelectiveScanCuda(torch.nn.Module):
    """Mamba selective scan (N = 16) on B200 with autograd.

    ``forward`` without ``h_prev`` uses :class:`SelectiveScanFnV2`; with ``h_prev`` (and
    ``forward_with_state`` always) the stateful :class:`SelectiveScanCudaFunction`. Both
    backward passes run on the GPU.
    """

    def __init__(self):
        super().__init__()
        self._module = None

    def _get_module(self):
        """The op module (mamba_cuda.py:1185-1188): the reference's five host entry points."""
        if self._module is None:
            self._module = _get_selective_scan_cuda_module()
        return self._module

    def forward(self, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
        if h_prev is not None:
            out, _ = SelectiveScanCudaFunction.apply(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
            return out
        return SelectiveScanFnV2.apply(u, delta, A, B_ssm, C_ssm, D_ssm)

    def forward_with_state(self, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
        """Returns ``(out (B, L, D), h_last (B, D, 16))``; ``h_prev`` seeds the state."""
        return SelectiveScanCudaFunction.apply(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)


# ---------------------------------------------------------------------------
# Plain PyTorch reference functions (API kept from the reference; not used by the
# CUDA path).
# ---------------------------------------------------------------------------

def selective_scan_ref(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None, return_intermediates=False):
    """PyTorch selective scan with autograd (any device / dtype).

    u, delta: (B, L, D); A: (D, N); B_ssm, C_ssm: (B, L, N); D_ssm: (D,);
    h_prev: (B, D, N) or None. Returns ``(out, h_last)`` and, when
    ``return_intermediates``, a dict with the keys of mamba_cuda.py:933-943
    (h_states, dA, dBu of shape (B, D, N, L), u_t, delta_t, B_t, C_t, h_prev) plus "A".
    The time axis of the per-step tensors is last, which is what the reference's
    time loop indexes (its einsum at :910 put the state axis there instead).
    """
    Bb, L, D = u.shape
    N = A.shape[1]
    u_t = u.transpose(1, 2)
    delta_t = delta.transpose(1, 2)
    B_t = B_ssm.transpose(1, 2)
    C_t = C_ssm.transpose(1, 2)
    if h_prev is None:
        h_prev = torch.zeros(Bb, D, N, device=u.device, dtype=u.dtype)
    dA = torch.exp(delta_t.unsqueeze(2) * A.unsqueeze(0).unsqueeze(-1))      # (B, D, N, L)
    dBu = (delta_t * u_t).unsqueeze(2) * B_t.unsqueeze(1)                    # (B, D, N, L)
    h = h_prev
    states = []
    for t in range(L):
        h = dA[..., t] * h + dBu[..., t]
        states.append(h)
    h_states = torch.stack(states, dim=-1) if states else h_prev.new_zeros(Bb, D, N, 0)
    y = (C_t.unsqueeze(1) * h_states).sum(dim=2) + u_t * D_ssm.view(1, -1, 1)
    out = y.transpose(1, 2)
    if return_intermediates:
        inter = {"h_states": h_states, "dA": dA, "dBu": dBu, "u_t": u_t, "delta_t": delta_t,
                 "B_t": B_t, "C_t": C_t, "h_prev": h_prev, "A": A}
        return out, h, inter
    return out, h


def selective_scan_backward(dout, dh_last, intermediates, D_ssm):
    """Gradients of ``selective_scan_ref`` from its intermediates (PyTorch, any device).

    Same signature and return order as the reference (mamba_cuda.py:949-1041):
    ``(du, ddelta, dA, dB_ssm, dC_ssm, dD_ssm, dh_prev)``; here every term is the exact
    derivative (the chain through exp(delta*A) included), with the A-gradient taken with
    respect to A itself. ``intermediates`` must carry "A" (``selective_scan_ref`` adds it).
    """
    hs = intermediates["h_states"]          # (B, D, N, L)
    dAe = intermediates["dA"]               # exp(delta*A), (B, D, N, L)
    u_t = intermediates["u_t"]
    delta_t = intermediates["delta_t"]
    B_t = intermediates["B_t"]
    C_t = intermediates["C_t"]
    h_prev = intermediates["h_prev"]
    Bb, D, N, L = hs.shape
    if "A" not in intermediates:
        raise KeyError("intermediates lack 'A'; produce them with selective_scan_ref("
                       "..., return_intermediates=True)")
    A = intermediates["A"].unsqueeze(0)     # (1, D, N)
    dout_t = dout.transpose(1, 2)
    q = dh_last.clone() if dh_last is not None else torch.zeros_like(h_prev)
    du = torch.zeros_like(u_t)
    ddelta = torch.zeros_like(delta_t)
    dA = torch.zeros(D, N, dtype=hs.dtype, device=hs.device)
    dB = torch.zeros_like(B_t)
    dC = torch.zeros_like(C_t)
    for t in range(L - 1, -1, -1):
        gy = dout_t[:, :, t]
        g = gy.unsqueeze(-1) * C_t[:, :, t].unsqueeze(1) + q
        hprev = hs[..., t - 1] if t > 0 else h_prev
        ah = dAe[..., t] * hprev
        dC[:, :, t] = (gy.unsqueeze(-1) * hs[..., t]).sum(1)
        dB[:, :, t] = (g * (delta_t[:, :, t] * u_t[:, :, t]).unsqueeze(-1)).sum(1)
        sgb = (g * B_t[:, :, t].unsqueeze(1)).sum(-1)
        du[:, :, t] = gy * D_ssm.view(1, -1) + delta_t[:, :, t] * sgb
        ddelta[:, :, t] = (g * ah * A).sum(-1) + u_t[:, :, t] * sgb
        dA = dA + (g * ah * delta_t[:, :, t].unsqueeze(-1)).sum(0)
        q = dAe[..., t] * g
    dD = (dout_t * u_t).sum(dim=(0, 2))
    return (du.transpose(1, 2), ddelta.transpose(1, 2), dA, dB.transpose(1, 2),
            dC.transpose(1, 2), dD, q)
