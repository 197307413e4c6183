"""Causal depthwise conv1d, the producer of the scan's input u in Mamba's block:
``causal_conv1d_fn(x, weight, bias=None, activation=None, x_prev=None)``.

Not in the reference (the official Mamba stack ships it as causal_conv1d). The layout is the
scan's channel-last one: x (B, L, D), weight (D, W) with W <= 4, bias (D); ``x_prev``
(B, W-1, D) holds the W-1 inputs before t = 0 for chunked streaming (zero when None), and
``x[:, -(W-1):]`` (see :func:`conv_state`) is the next chunk's ``x_prev``.

    y[b, t, d] = act(bias[d] + sum_k weight[d, k] * x[b, t - (W-1) + k, d]),  act in {None, "silu"}

Forward and backward run on the GPU (mwc_conv1d_fwd / mwc_conv1d_bwd).
"""
from __future__ import annotations

import torch

from . import _lib
from ._ops import _on_device, _p, _stream, dtype_code

__all__ = ["CausalConv1dFn", "causal_conv1d_fn", "causal_conv1d_ref", "conv_state"]

_ACT = {None: 0, "silu": 1, "swish": 1}


def _check(x, weight, bias, x_prev, activation):
    if activation not in _ACT:
        raise RuntimeError("activation must be None or 'silu'")
    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dim() == 3):
        raise RuntimeError("x must be a CUDA tensor (batch, seqlen, dim)")
    Bb, L, D = x.shape
    if weight.dim() != 2 or weight.shape[0] != D or not 1 <= weight.shape[1] <= 4:
        raise RuntimeError("weight must be (dim, width) with 1 <= width <= 4")
    W = weight.shape[1]
    for name, t, shape in (("weight", weight, None), ("bias", bias, (D,)),
                           ("x_prev", x_prev, (Bb, W - 1, D))):
        if t is None:
            continue
        if t.dtype != x.dtype or t.device != x.device:
            raise RuntimeError(f"{name} must match x in dtype and device")
        if shape is not None and tuple(t.shape) != shape:
            raise RuntimeError(f"{name} must have shape {shape}")
    dtype_code(x)


class CausalConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias=None, activation=None, x_prev=None):
        _check(x, weight, bias, x_prev, activation)
        x, weight = x.contiguous(), weight.contiguous()
        bias = bias.contiguous() if bias is not None else None
        x_prev = x_prev.contiguous() if x_prev is not None else None
        Bb, L, D = x.shape
        W = weight.shape[1]
        y = torch.empty_like(x)
        lib = _lib.load()
        with _on_device(x.device):
            rc = lib.mwc_conv1d_fwd(_p(x), _p(weight), _p(bias), _p(x_prev), _ACT[activation], _p(y),
                                    Bb, L, D, W, dtype_code(x), _stream(x.device))
        _lib.check(rc, "causal_conv1d forward")
        ctx.save_for_backward(x, weight, bias, x_prev)
        ctx.act = _ACT[activation]
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, bias, x_prev = ctx.saved_tensors
        Bb, L, D = x.shape
        W = weight.shape[1]
        dy = dy.contiguous()
        dx = torch.empty_like(x)
        dw = torch.empty_like(weight)
        db = torch.empty_like(bias) if bias is not None else None
        dxp = torch.empty_like(x_prev) if x_prev is not None and ctx.needs_input_grad[4] else None
        lib = _lib.load()
        with _on_device(x.device):
            ws_bytes = int(lib.mwc_conv1d_bwd_workspace_bytes(Bb, L, D, W))
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
            rc = lib.mwc_conv1d_bwd(_p(x), _p(weight), _p(bias), _p(x_prev), ctx.act, _p(dy), _p(dx),
                                    _p(dw), _p(db), _p(dxp), _p(ws), ws_bytes, Bb, L, D, W,
                                    dtype_code(x), _stream(x.device))
        _lib.check(rc, "causal_conv1d backward")
        return dx, dw, db, None, dxp


def causal_conv1d_fn(x, weight, bias=None, activation=None, x_prev=None):
    """Causal depthwise conv1d over time of a (B, L, D) tensor (see the module docstring)."""
    return CausalConv1dFn.apply(x, weight, bias, activation, x_prev)


def conv_state(x, width, x_prev=None):
    """The last width-1 inputs (B, width-1, D) of x (preceded by x_prev when x is shorter):
    the x_prev of the next chunk."""
    if width <= 1:
        return x[:, :0]
    full = torch.cat([x_prev, x], dim=1) if x_prev is not None else x
    if full.shape[1] < width - 1:
        pad = torch.zeros(x.shape[0], width - 1 - full.shape[1], x.shape[2], dtype=x.dtype, device=x.device)
        full = torch.cat([pad, full], dim=1)
    return full[:, -(width - 1):]


def causal_conv1d_ref(x, weight, bias=None, activation=None, x_prev=None):
    """Plain PyTorch version of :func:`causal_conv1d_fn` (any device / dtype, autograd)."""
    Bb, L, D = x.shape
    W = weight.shape[1]
    if x_prev is None:
        x_prev = torch.zeros(Bb, W - 1, D, dtype=x.dtype, device=x.device)
    full = torch.cat([x_prev, x], dim=1)                       # (B, W-1+L, D)
    y = sum(weight[:, k] * full[:, k:k + L] for k in range(W))
    if bias is not None:
        y = y + bias
    if activation in ("silu", "swish"):
        y = torch.nn.functional.silu(y)
    return y
