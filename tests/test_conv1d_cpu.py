"""Causal conv1d checker on CPU: the plain-PyTorch causal_conv1d_ref against an explicit
float64 loop of the definition, its autograd against finite differences (gradcheck), and
the streaming property (two chunks joined through conv_state / x_prev = one call)."""
import numpy as np
import pytest
import torch

from mamba_windows_cuda.causal_conv1d import causal_conv1d_ref, conv_state


def loop_conv(x, w, b, act, x_prev):
    """y[b,t,d] = act(bias[d] + sum_k w[d,k] x[b, t-(W-1)+k, d]), x[t<0] from x_prev / 0."""
    B, L, D = x.shape
    W = w.shape[1]
    xp = np.zeros((B, W - 1, D)) if x_prev is None else x_prev
    full = np.concatenate([xp, x], axis=1)
    y = np.zeros((B, L, D))
    for t in range(L):
        for k in range(W):
            y[:, t, :] += w[:, k][None, :] * full[:, t + k, :]
    if b is not None:
        y += b[None, None, :]
    if act == "silu":
        y = y / (1.0 + np.exp(-y))
    return y


@pytest.mark.parametrize("W", [1, 2, 3, 4])
@pytest.mark.parametrize("act", [None, "silu"])
@pytest.mark.parametrize("with_prev", [False, True])
def test_ref_matches_loop(W, act, with_prev):
    g = torch.Generator().manual_seed(W)
    x = torch.randn(2, 17, 5, generator=g, dtype=torch.float64)
    w = torch.randn(5, W, generator=g, dtype=torch.float64)
    b = torch.randn(5, generator=g, dtype=torch.float64)
    xp = torch.randn(2, W - 1, 5, generator=g, dtype=torch.float64) if with_prev else None
    y = causal_conv1d_ref(x, w, b, act, xp)
    ref = loop_conv(x.numpy(), w.numpy(), b.numpy(), act, xp.numpy() if xp is not None else None)
    assert np.abs(y.numpy() - ref).max() < 1e-12


def test_ref_gradcheck():
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 9, 3, generator=g, dtype=torch.float64, requires_grad=True)
    w = torch.randn(3, 4, generator=g, dtype=torch.float64, requires_grad=True)
    b = torch.randn(3, generator=g, dtype=torch.float64, requires_grad=True)
    xp = torch.randn(2, 3, 3, generator=g, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda *a: causal_conv1d_ref(*a[:3], "silu", a[3]), (x, w, b, xp))


def test_streaming_chunks_equal_one_call():
    g = torch.Generator().manual_seed(8)
    x = torch.randn(2, 40, 6, generator=g, dtype=torch.float64)
    w = torch.randn(6, 4, generator=g, dtype=torch.float64)
    y = causal_conv1d_ref(x, w, None, "silu")
    y1 = causal_conv1d_ref(x[:, :25], w, None, "silu")
    y2 = causal_conv1d_ref(x[:, 25:], w, None, "silu", conv_state(x[:, :25], 4))
    assert torch.allclose(torch.cat([y1, y2], 1), y, atol=1e-12)
