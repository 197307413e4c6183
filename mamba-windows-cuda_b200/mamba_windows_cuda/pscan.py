"""First-order linear recurrence scan: drop-in for mamba_windows_cuda/pscan.py.

``parallel_scan_fn(A, X)`` computes ``H_0 = X_0``, ``H_t = A_t H_{t-1} + X_t`` along
dim 2 of (B, D, L, N) tensors with autograd, on the sm_100a kernel of libmwc_b200.so (one
pass over memory; any L, not only powers of two). ``parallel_scan_ref`` is the plain
sequential PyTorch loop of the reference (pscan.py:153-171) and runs on any device.

The reference's ``PScan`` Blelloch sweeps (pscan.py:16-136) are replaced; the class name
is kept as the autograd Function.
"""
from __future__ import annotations

import torch

from . import _ops


def _check(A, X):
    for name, t in (("A", A), ("X", X)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    if X.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise RuntimeError("X must be float32/float16/bfloat16")
    if A.dtype != X.dtype:
        raise RuntimeError("A dtype must match X dtype")
    if X.dim() != 4 or A.shape != X.shape:
        raise RuntimeError("A and X must both be (B, D, L, N) with the same shape")
    if A.device != X.device:
        raise RuntimeError("A and X must be on the same device")


class PScan(torch.autograd.Function):
    """Autograd Function of the linear recurrence (forward and backward on the GPU).

    Backward: gX_t = g_t + A_{t+1} gX_{t+1}, gA_t = gX_t H_{t-1} (gA_0 = 0).
    """

    @staticmethod
    def forward(ctx, A_in, X_in):
        _check(A_in, X_in)
        A = A_in.contiguous()
        X = X_in.contiguous()
        H = _ops.lin_scan_forward(A, X)
        ctx.save_for_backward(A, H)
        return H

    @staticmethod
    def backward(ctx, grad_output):
        A, H = ctx.saved_tensors
        gA, gX = _ops.lin_scan_backward(A, H, grad_output.contiguous())
        return gA, gX


def parallel_scan_fn(A, X):
    """H[t] = A[t] * H[t-1] + X[t] along dim 2 of (B, D, L, N); H[0] = X[0]."""
    return PScan.apply(A, X)


def parallel_scan_ref(A, X):
    """Sequential reference scan (any device / dtype), same semantics as parallel_scan_fn."""
    B, D, L, N = A.shape
    H = torch.zeros_like(X)
    if L == 0:
        return H
    H[:, :, 0] = X[:, :, 0]
    for t in range(1, L):
        H[:, :, t] = A[:, :, t] * H[:, :, t - 1] + X[:, :, t]
    return H
