"""Shared input generators and tolerance checks for the tests (CPU and GPU)."""
from __future__ import annotations

import numpy as np
import torch

N = 16


def rel_err(x, ref) -> float:
    """Normwise relative error max|x - ref| / max|ref| (the 'max relative error' of the
    fp32 tolerance; an elementwise ratio is meaningless at zero crossings)."""
    x = np.asarray(x.detach().cpu().double() if isinstance(x, torch.Tensor) else x, np.float64)
    ref = np.asarray(ref.detach().cpu().double() if isinstance(ref, torch.Tensor) else ref,
                     np.float64)
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


def assert_fp32(x, ref, tol=1e-4, what=""):
    e = rel_err(x, ref)
    assert e < tol, f"{what}: normwise relative error {e:.3e} >= {tol}"


def assert_fp16(x, ref, what="", atol=2e-2, rtol=1e-2):
    """fp16 tolerance atol 2e-2 / rtol 1e-2, elementwise, against a float64 result."""
    x = x.detach().cpu().double().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(x - ref) > atol + rtol * np.abs(ref)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} elements outside "
                           f"atol {atol} / rtol {rtol}; max abs err {np.abs(x - ref).max():.3e}")


def make_inputs(B, L, D, dtype=torch.float32, seed=0, dist="c1", with_state=False,
                device="cpu"):
    """Seeded inputs with BASELINE.json's distributions.

    dist "c1"/"c3": u~N(0,1), delta=softplus(N(-1,.5)), A=-(n+1), B,C~N(0,1), D=1
    dist "c2": delta=softplus(N(-2,.5)), A=-(n+1)(1+0.1U), B,C~N(0,1)/4, D~U(.5,1.5)
    dist "c4": delta=softplus(N(-3,.5)), A=-(n+1)/16, B,C~N(0,1), D=1
    dist "reftest": the reference tests' u~0.1N, delta=0.01, A=-0.1U, B,C~0.1N, D=0.1
    Also returns g~N(0,1) (B,L,D), and h_prev / gh (B,D,16) when with_state.
    """
    g = torch.Generator().manual_seed(seed)
    f = torch.float32
    n1 = torch.arange(1, N + 1, dtype=f)
    if dist in ("c1", "c3"):
        u = torch.randn(B, L, D, generator=g)
        delta = torch.nn.functional.softplus(torch.randn(B, L, D, generator=g) * 0.5 - 1.0)
        A = -n1.repeat(D, 1)
        Bm = torch.randn(B, L, N, generator=g)
        Cm = torch.randn(B, L, N, generator=g)
        Dv = torch.ones(D)
    elif dist == "c2":
        u = torch.randn(B, L, D, generator=g)
        delta = torch.nn.functional.softplus(torch.randn(B, L, D, generator=g) * 0.5 - 2.0)
        A = -n1.repeat(D, 1) * (1 + 0.1 * torch.rand(D, N, generator=g))
        Bm = torch.randn(B, L, N, generator=g) / 4
        Cm = torch.randn(B, L, N, generator=g) / 4
        Dv = 0.5 + torch.rand(D, generator=g)
    elif dist == "c4":
        u = torch.randn(B, L, D, generator=g)
        delta = torch.nn.functional.softplus(torch.randn(B, L, D, generator=g) * 0.5 - 3.0)
        A = -(n1 / 16).repeat(D, 1)
        Bm = torch.randn(B, L, N, generator=g)
        Cm = torch.randn(B, L, N, generator=g)
        Dv = torch.ones(D)
    elif dist == "reftest":
        u = torch.randn(B, L, D, generator=g) * 0.1
        delta = torch.full((B, L, D), 0.01)
        A = -torch.rand(D, N, generator=g) * 0.1
        Bm = torch.randn(B, L, N, generator=g) * 0.1
        Cm = torch.randn(B, L, N, generator=g) * 0.1
        Dv = torch.full((D,), 0.1)
    else:
        raise ValueError(dist)
    gy = torch.randn(B, L, D, generator=g)
    hp = torch.randn(B, D, N, generator=g) * (0.1 if dist == "c3" else 1.0) if with_state else None
    gh = torch.randn(B, D, N, generator=g) if with_state else None
    cast = (lambda t: None if t is None else t.to(dtype).to(device))
    return {k: cast(v) for k, v in dict(u=u, delta=delta, A=A, Bm=Bm, Cm=Cm, Dv=Dv, g=gy,
                                         h_prev=hp, gh=gh).items()}


def np64(t):
    return None if t is None else t.detach().cpu().double().numpy()
